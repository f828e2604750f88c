// sa_common.cuh — shared definitions for the sparse_attn sm_100a kernels.
//
// Problem (track-01/reference/reference.py:10-40): for every query row
// (b, m) and every head h of 16,
//   o[b,m,h,:] = sum_t softmax_t([s_0..s_{topk-1}, sink[h]]) * kv[b, idx[b,m,t], :]
//   s_t = scale * <q[b,m,h,:], kv[b, idx[b,m,t], :]>
// with K == V (one shared 512-wide row per slot).  Slots with idx == -1 are
// masked (track-01/submission.py:313-322); here every idx outside
// [0, kv_len) is masked, so the kernels never read out of bounds.
//
// Work schedule ("units"): the flattened (row, key-block) space.  A query
// row ("token") has `upt` = ceil(topk / UNIT_KEYS) units of UNIT_KEYS slots.
// The U = tokens * upt units are cut into `grid` contiguous, equal ranges,
// one per persistent CTA: CTA g owns [g*U/grid, (g+1)*U/grid).  A CTA's range
// may cross any number of token boundaries; each maximal piece of one token
// inside one CTA is a "segment".  A segment that covers
// its whole token writes the bf16 output directly; a segment that covers only
// part of its token (at most the first and the last segment of a CTA) writes
// an fp32 partial (unnormalised O, running max, running sum) into workspace
// slot 2g (first segment) or 2g+1 (last segment), and a combine kernel merges
// the partials of each split token.  This balances the gather load across all
// SMs whatever (b*m, topk) is, which the reference's one-program-per-token
// grid (submission.py:1005) does not.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace sa {

constexpr int kHeads = 16;
constexpr int kDim = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* kv;
  const float* sink;
  const int32_t* idx;
  __nv_bfloat16* o;
  int64_t b, m, kv_len, topk;
  int64_t q_sb, q_sm, q_sh;  // element strides, d stride is 1
  int64_t kv_sb, kv_sn;
  int64_t i_sb, i_sm, i_sk;
  int64_t o_sb, o_sm, o_sh;
  float scale_log2;  // scale * log2(e): scores are kept in the log2 domain
  float* part_acc;   // [2*grid][16][512] fp32 unnormalised partial O
  float* part_ml;    // [2*grid][2][16]   running max (log2 domain), running sum
  int64_t upt;       // units per token
  int64_t units;     // tokens * upt
  int grid;
  // fp8 KV cache only (sa_fwd_fp8): kv holds e4m3 bytes (kv_sb, kv_sn in
  // bytes) and row t of batch b dequantises as kv8[b,t,:] * kscale[b,t]
  const float* kscale;
  int64_t ks_sb, ks_sn;
  // One word per CTA (workspace, zero between calls): the number of CTAs that
  // finished their part of the row split at the start of CTA f's range.  The
  // last one merges the row and zeroes the word again (sa_ws.cu).
  int* tickets;
  int merge_in_kernel;  // sa_ws only: merge split rows by ticket instead of the combine kernel
  // Optional (sa_fwd_train, ws kernel): lse[row][h] = log2 of the row's full
  // softmax denominator, the sink included, in the log2 domain of the scores
  // (p_t = 2^(s_t * scale * log2(e) - lse)); the backward pass reads it.
  float* lse;
  int64_t lse_rs;  // floats between lse rows (the caller's head count)
  // Optional (ws kernel, many rows): units to run per row, written by
  // sa_row_units_kernel; set, each CTA runs whole rows of a fixed snake
  // order instead of a contiguous unit range (sa_ws.cu).
  const int* row_units;
  // Polls before a pipeline wait gives up (sa_set_option(SA_OPT_SPIN_LIMIT));
  // test_stall != 0 withholds one arrival on the first ring slot so that a
  // wait runs out (the failure-path test, SA_OPT_TEST_STALL).
  uint32_t spin;
  int test_stall;
  // L2 policy of the KV row gathers: 0 evict_first, 1 evict_normal,
  // 2 evict_last (l2_policy_kv)
  int kv_policy;
  // Head groups of 16 run by one launch (ws kernel; 1 elsewhere): group
  // blockIdx.y reads heads 16y..16y+15 of q (the Q map spans all hg * 16) and
  // writes them in o and lse; its CTAs use workspace slots and tickets
  // [y * grid, (y + 1) * grid).  The groups' CTAs with one blockIdx.x walk the
  // same units at the same time, so a KV row gathered for one group is an L2
  // hit for the others.
  int hg;
};

// Process-wide options (sa_set_option, sa_abi.cu).
bool opt_row_schedule();
bool opt_indexer_tc();
uint32_t opt_spin_limit();
int opt_test_stall();
int opt_kv_policy();  // -1: by the call's reuse (sa_abi.cu)
bool opt_gather_only();

// log2 of the full denominator for a running max m and sum l (relative to m),
// with the sink as the extra logit; all in the log2 domain.
__device__ __forceinline__ float row_lse2(float m_run, float l_run, float sink_log2) {
  const float M = fmaxf(m_run, sink_log2);
  const float den = (m_run == -INFINITY ? 0.f : l_run * exp2f(m_run - M)) + exp2f(sink_log2 - M);
  return M + log2f(den);
}

// Workspace layout shared by the host (sizing) and the kernels.
constexpr size_t kPartAccFloats = (size_t)kHeads * kDim;
constexpr size_t kPartMlFloats = 2 * kHeads;

// The Params of head group y (see Params::hg): output, sink, lse and
// workspace pointers moved to the group's heads and slots.
__device__ __forceinline__ Params group_params(const Params& p, int y) {
  Params r = p;
  const int64_t gb = (int64_t)y * p.grid;
  r.o += (int64_t)y * kHeads * p.o_sh;
  r.sink += y * kHeads;
  if (r.lse != nullptr) r.lse += y * kHeads;
  r.part_acc += 2 * gb * kPartAccFloats;
  r.part_ml += 2 * gb * kPartMlFloats;
  r.tickets += gb;
  return r;
}

__host__ __device__ constexpr size_t ws_acc_bytes(int grid) {
  return ((size_t)2 * grid * kPartAccFloats * sizeof(float) + 255) & ~(size_t)255;
}
__host__ __device__ constexpr size_t ws_ml_bytes(int grid) {
  return ((size_t)2 * grid * kPartMlFloats * sizeof(float) + 255) & ~(size_t)255;
}
// The ticket words come first, at a fixed offset and sized for the largest
// grid, so that calls with different grids never find partial data where
// another call's tickets are expected to be zero.
constexpr int kMaxGrid = 512;  // >= 2 x the SM count of any supported device
constexpr size_t kTicketBytes = kMaxGrid * sizeof(int);
__host__ __device__ constexpr size_t workspace_bytes_for_grid(int grid) {
  return kTicketBytes + ws_acc_bytes(grid) + ws_ml_bytes(grid);
}

// Row-unit counts (one int per row) after the partials, for the row schedule.
__host__ __device__ constexpr size_t row_units_bytes(int64_t rows) {
  return ((size_t)rows * sizeof(int) + 255) & ~(size_t)255;
}

__host__ __device__ inline int64_t unit_begin(int64_t g, int64_t units, int64_t grid) {
  return (g * units) / grid;
}

// Largest CTA index k with unit_begin(k) <= u (requires grid <= units).
__host__ __device__ inline int64_t cta_of_unit(int64_t u, int64_t units, int64_t grid) {
  return ((u + 1) * grid - 1) / units;
}

// Row schedule (many rows, p.row_units set): CTA g runs whole rows, the
// positions g, 2G-1-g, 2G+g, 4G-1-g, ... of the rows taken in descending
// index order (snake rounds of G).  Every thread derives the same sequence.
// When the costs fall along the row index (causal prefill, where row i holds
// min(i+1, topk) slots followed by -1 padding) the rounds pair long rows
// with short ones; equal rows get an equal share of rows.
__device__ __forceinline__ int64_t snake_row(int64_t k, int64_t g, int64_t G, int64_t R) {
  const int64_t pos = k * G + ((k & 1) ? (G - 1 - g) : g);
  return pos < R ? R - 1 - pos : -1;
}
__device__ __forceinline__ int64_t units_of_row(const Params& p, int64_t r) {
  return r >= 0 ? __ldg(p.row_units + r) : 0;
}

// A producer's place in the row schedule: row t (batch tb, row tm within
// it), unit kb of its nu_t units; the next row's count is loaded a row ahead.
struct RowCursor {
  int64_t kb, tb, tm, t, sk, nu_t, nu_n;
  __device__ __forceinline__ void start(const Params& p, int64_t g, int64_t G, int64_t R) {
    sk = 0;
    kb = 0;
    t = snake_row(0, g, G, R);
    tb = t / p.m;
    tm = t - tb * p.m;
    nu_t = units_of_row(p, t);
    nu_n = units_of_row(p, snake_row(1, g, G, R));
  }
  __device__ __forceinline__ void advance(const Params& p, int64_t g, int64_t G, int64_t R) {
    if (++kb == nu_t) {
      kb = 0;
      t = snake_row(++sk, g, G, R);
      tb = t / p.m;
      tm = t - tb * p.m;
      nu_t = nu_n;
      nu_n = units_of_row(p, snake_row(sk + 1, g, G, R));
    }
  }
};

// Writes p.row_units for the row schedule (sa_ws.cu; any forward kernel
// with a kRows instance runs after it in the same stream).
cudaError_t launch_row_units(const Params& p, cudaStream_t st);

// Runs `fn` (returning cudaError_t) once per CUDA device, the first time it is
// called with that device current; later calls return the first result.
struct PerDeviceOnce {
  static constexpr int kMax = 64;
  std::once_flag flag[kMax];
  cudaError_t err[kMax] = {};
};
template <class Fn>
cudaError_t once_per_device(PerDeviceOnce& o, Fn&& fn) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= PerDeviceOnce::kMax) return cudaErrorInvalidDevice;
  std::call_once(o.flag[dev], [&] { o.err[dev] = fn(); });
  return o.err[dev];
}

// Launches the LSE-combine kernel when some row is split across CTAs
// (defined in sa_mma.cu, shared by every variant).
cudaError_t launch_combine(const Params& p, cudaStream_t st);

// ----------------------------------------------------------------------------
// PTX wrappers (sm_80+ instructions that remain the right tool on sm_100a for
// scattered 16-byte row gathers and register-level bf16 MMA).
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async copy global->shared; src_bytes == 0 zero-fills without reading.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async16_hint(uint32_t dst, const void* src, int src_bytes,
                                                uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;\n" ::"r"(dst),
               "l"(src), "r"(src_bytes), "l"(policy)
               : "memory");
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}

// L2 policy of the KV row gathers (Params::kv_policy): rows that no other
// query row of the call will read are best evicted first; rows that many
// query rows share (prefill: m * topk >= kv_len) are kept.
__device__ __forceinline__ uint64_t l2_policy_kv(int kv_policy) {
  uint64_t p;
  if (kv_policy == 2) {
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
  } else if (kv_policy == 1) {
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;\n" : "=l"(p));
  } else {
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  }
  return p;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ bool slot_valid(int64_t key, int64_t topk, int32_t id,
                                           int64_t kv_len) {
  return key < topk && id >= 0 && (int64_t)id < kv_len;
}

// An index that is neither the -1 sentinel nor inside [0, kv_len) is masked
// like -1 but also counted: each kernel's translation unit keeps a device
// counter of such slots (read and reset by sa_index_faults), so a caller can
// tell its index producer wrote garbage.  Warp-aggregated: one atomic per
// unit that holds any.
__device__ __forceinline__ bool index_fault(int32_t id, int64_t kv_len) {
  return id < -1 || (int64_t)id >= kv_len;
}
__device__ __forceinline__ void count_index_faults(unsigned long long* counter, uint32_t n) {
  if (n != 0u) atomicAdd(counter, (unsigned long long)n);
}
// Host side: read (and optionally zero) one translation unit's counter.
template <typename Sym>
inline int index_fault_io(const Sym& sym, unsigned long long* out, bool reset) {
  unsigned long long v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, sym, sizeof(v));
  if (e == cudaSuccess && reset) {
    const unsigned long long zero = 0;
    e = cudaMemcpyToSymbol(sym, &zero, sizeof(zero));
  }
  if (e != cudaSuccess) return (int)e;
  *out += v;
  return 0;
}

// Final normalisation with the sink as the (topk+1)-th logit
// (track-01/reference/reference.py:34-38, submission.py:340-345): the sink adds
// exp(sink - max) to the denominator and nothing to the numerator.
// m_run is the running max in the log2 domain (-inf when no slot was valid),
// l_run the running sum of exp2(s - m_run).  Returns the factor that turns the
// unnormalised accumulator into o.
__device__ __forceinline__ float sink_factor(float m_run, float l_run, float sink_log2) {
  float M = fmaxf(m_run, sink_log2);
  float alpha = exp2f(m_run - M);  // 0 when m_run == -inf
  float den = l_run * alpha + exp2f(sink_log2 - M);
  return alpha / den;
}

// Merge of a split row: head h, columns d0..d0+7 of row t, whose units
// CTAs f..f+np-1 computed; the fp32 partials are combined with the sink as the
// extra logit (reference.py:34-38) and o is written in bf16.  Partial k of the
// row sits in slot 2(f+k), except k = 0 when the row starts inside CTA f's
// range (f_mid): that is f's last segment, slot 2f+1.  All loads of a batch of
// up to kCombineBatch partials are issued together: one memory round trip.
constexpr int kCombineBatch = 4;
__device__ __forceinline__ void merge_split_row(const Params& p, int64_t f, int np, bool f_mid,
                                                int64_t t, int h, int d0) {
  auto slot_of = [&](int k) -> int64_t { return (k == 0 && f_mid) ? 2 * f + 1 : 2 * (f + k); };
  const float sink_l2 = __ldg(p.sink + h) * kLog2e;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  float M = sink_l2, den = 1.f;  // den relative to M (= exp2(sink - M) for M = sink)
  for (int k0 = 0; k0 < np; k0 += kCombineBatch) {
    float mk[kCombineBatch], lk[kCombineBatch];
    float4 va[kCombineBatch], vb[kCombineBatch];
#pragma unroll
    for (int k = 0; k < kCombineBatch; ++k) {
      mk[k] = -INFINITY;
      lk[k] = 0.f;
      va[k] = vb[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + k < np) {
        const int64_t sl = slot_of(k0 + k);
        mk[k] = __ldcg(p.part_ml + sl * kPartMlFloats + h);
        lk[k] = __ldcg(p.part_ml + sl * kPartMlFloats + kHeads + h);
        const float4* src =
            reinterpret_cast<const float4*>(p.part_acc + sl * kPartAccFloats + h * kDim + d0);
        va[k] = __ldcg(src);
        vb[k] = __ldcg(src + 1);
      }
    }
    float Mb = M;
#pragma unroll
    for (int k = 0; k < kCombineBatch; ++k) Mb = fmaxf(Mb, mk[k]);
    const float r = exp2f(M - Mb);  // rescale what was merged so far
    den *= r;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] *= r;
#pragma unroll
    for (int k = 0; k < kCombineBatch; ++k) {
      const float w = exp2f(mk[k] - Mb);  // 0 for absent partials
      den += lk[k] * w;
      acc[0] += w * va[k].x;
      acc[1] += w * va[k].y;
      acc[2] += w * va[k].z;
      acc[3] += w * va[k].w;
      acc[4] += w * vb[k].x;
      acc[5] += w * vb[k].y;
      acc[6] += w * vb[k].z;
      acc[7] += w * vb[k].w;
    }
    M = Mb;
  }
  const float inv = 1.f / den;
  if (p.lse != nullptr && d0 == 0) p.lse[t * p.lse_rs + h] = M + log2f(den);
  const int64_t tb = t / p.m, tm = t - tb * p.m;
  uint4 w;
  w.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  w.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  w.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
  w.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
  *reinterpret_cast<uint4*>(p.o + tb * p.o_sb + tm * p.o_sm + h * p.o_sh + d0) = w;
}


}  // namespace sa
