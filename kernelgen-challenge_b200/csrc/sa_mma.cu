// sa_mma.cu — persistent gather-attend kernel on the warp-level bf16 MMA path
// (mma.sync m16n8k16) with a cp.async gather ring, plus the LSE-combine kernel
// shared by every variant.
//
// Algorithm (track-01/submission.py:276-347, the reference's NVIDIA-path
// "universal" kernel; math of track-01/reference/reference.py:24-40):
//   for each key block of one query row:
//     S = Q K^T * scale           (16 heads x keys, fp32)
//     S[masked] = -inf            (submission.py:313-322)
//     online softmax update       (submission.py:324-338)
//     O = O * corr + P(bf16) V    (submission.py:333-335)
//   o = O / (l + exp(sink - max)) (submission.py:340-345)
//
// B200 mapping (one persistent CTA per SM, 8 warps):
//   * the CTA walks its contiguous range of (row, 32-key unit) work
//     (see sa_common.cuh) through a 4-deep ring of 32 x 1 KiB gathered rows;
//     indices run 6 units ahead of the rows through their own cp.async ring,
//     so no load ever waits on another load;
//   * warp w owns head-dim columns [64w, 64w+64): it computes the partial
//     scores of those columns for all 16 heads x 32 keys (Q slice in
//     registers), the 8 partials are summed through shared memory, 256
//     threads run the online softmax (16 threads per head), and each warp
//     then accumulates P V for its own 64 columns (O in registers);
//   * smem rows are XOR-swizzled in 16-byte chunks so both ldmatrix and
//     ldmatrix.trans read conflict-free;
//   * a 32-key unit whose slots are all masked is skipped (no loads were
//     issued for it either: masked rows are zero-filled without reading).
#include "sa_common.cuh"

namespace sa {

__device__ unsigned long long sa_mma_index_faults;  // out-of-range indices seen

namespace mma_path {

constexpr int BN = 32;      // keys per unit
constexpr int STAGES = 4;   // gathered-row ring depth
constexpr int IDXR = 8;     // index ring depth (>= 2*STAGES - 1)
constexpr int NWARP = 8;
constexpr int NT = NWARP * 32;
constexpr int RED_LD = 40;  // padded fp32 row of the score-reduction buffer
constexpr int P_LD = 40;    // padded bf16 row of the probability tile

struct Smem {
  __nv_bfloat16 kv[STAGES][BN][kDim];  // 128 KiB
  float red[NWARP][kHeads][RED_LD];    // 20 KiB
  __nv_bfloat16 p[kHeads][P_LD];
  int32_t idx[IDXR][BN];
  float corr[kHeads];
  float mrun[kHeads];
  float lrun[kHeads];
};

__device__ __forceinline__ uint32_t ldg32(const __nv_bfloat16* ptr) {
  return __ldg(reinterpret_cast<const unsigned int*>(ptr));
}

__global__ void __launch_bounds__(NT, 1) sa_mma_fwd_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, q4 = lane & 3;
  const int64_t G = p.grid, g = blockIdx.x;
  const int64_t u0 = unit_begin(g, p.units, G);
  const int64_t u1 = unit_begin(g + 1, p.units, G);
  const int n = static_cast<int>(u1 - u0);
  if (n <= 0) return;
  const int64_t upt = p.upt;
  const int64_t t_first = u0 / upt, t_last = (u1 - 1) / upt;
  const uint64_t pol = l2_policy_evict_first();

  // ---- producers -----------------------------------------------------------
  auto issue_idx = [&](int v) {
    if (warp == 0 && v < n) {
      const int64_t u = u0 + v, t = u / upt, kb = u - t * upt;
      const int64_t key = kb * BN + lane;
      const int64_t tb = t / p.m, tm = t - tb * p.m;
      const bool in = key < p.topk;
      const int32_t* src = p.idx + tb * p.i_sb + tm * p.i_sm + (in ? key : 0) * p.i_sk;
      cp_async4(smem_u32(&S.idx[v % IDXR][lane]), src, in ? 4 : 0);
    }
  };
  auto issue_kv = [&](int v) {
    if (v < n) {
      const int64_t u = u0 + v, t = u / upt, kb = u - t * upt;
      const __nv_bfloat16* base = p.kv + (t / p.m) * p.kv_sb;
      const int c = tid & 63, r0 = tid >> 6;
      const uint32_t dst0 = smem_u32(&S.kv[v % STAGES][0][0]);
#pragma unroll
      for (int k = 0; k < BN / 4; ++k) {
        const int r = r0 + 4 * k;
        const int32_t id = S.idx[v % IDXR][r];
        const bool ok = slot_valid(kb * BN + r, p.topk, id, p.kv_len);
        const __nv_bfloat16* src = base + (ok ? (int64_t)id : 0) * p.kv_sn + c * 8;
        cp_async16_hint(dst0 + r * (kDim * 2) + ((c ^ (r & 7)) << 4), src, ok ? 16 : 0, pol);
      }
    }
  };
  auto load_q = [&](int64_t t, uint32_t (&qa)[4][4]) {
    const int64_t tb = t / p.m, tm = t - tb * p.m;
    const __nv_bfloat16* qb = p.q + tb * p.q_sb + tm * p.q_sm;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int d0 = 64 * warp + 16 * ks + 2 * q4;
      qa[ks][0] = ldg32(qb + g8 * p.q_sh + d0);
      qa[ks][1] = ldg32(qb + (g8 + 8) * p.q_sh + d0);
      qa[ks][2] = ldg32(qb + g8 * p.q_sh + d0 + 8);
      qa[ks][3] = ldg32(qb + (g8 + 8) * p.q_sh + d0 + 8);
    }
  };

  uint32_t qn[4][4];
  load_q(t_first, qn);

  // ---- prologue: indices of the first 2*STAGES-2 units, rows of STAGES-1 ----
  for (int v = 0; v < 2 * STAGES - 2; ++v) issue_idx(v);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  for (int v = 0; v < STAGES - 1; ++v) {
    issue_kv(v);
    cp_async_commit();
  }

  // softmax-thread mapping: head sh, keys 2*sj and 2*sj+1 of the unit
  const int sh = tid >> 4, sj = tid & 15;
  float m_run = -INFINITY, l_run = 0.f;
  uint32_t qa[4][4];
  float o[8][4];
  int64_t seg_kb0 = 0;

  for (int i = 0; i < n; ++i) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();  // unit i's rows and unit i+STAGES-1's indices are visible
    issue_kv(i + STAGES - 1);
    issue_idx(i + 2 * STAGES - 2);
    cp_async_commit();

    const int64_t u = u0 + i, t = u / upt, kb = u - t * upt;
    const bool seg_start = (i == 0) || kb == 0;
    const bool seg_end = (i == n - 1) || kb == upt - 1;
    if (seg_start) {
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b2 = 0; b2 < 4; ++b2) qa[a][b2] = qn[a][b2];
      if (t < t_last) load_q(t + 1, qn);
#pragma unroll
      for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b2 = 0; b2 < 4; ++b2) o[a][b2] = 0.f;
      m_run = -INFINITY;
      l_run = 0.f;
      seg_kb0 = kb;
    }

    // validity of the unit's 32 slots (identical in every warp)
    const int32_t my_id = S.idx[i % IDXR][lane];
    const uint32_t vmask =
        __ballot_sync(0xffffffffu, slot_valid(kb * BN + lane, p.topk, my_id, p.kv_len));
    if (warp == 0) {
      const uint32_t f =
          __ballot_sync(0xffffffffu, kb * BN + lane < p.topk && index_fault(my_id, p.kv_len));
      if (lane == 0) count_index_faults(&sa_mma_index_faults, __popc(f));
    }

    if (vmask != 0u) {
      const uint32_t kvs = smem_u32(&S.kv[i % STAGES][0][0]);
      // ---- partial scores over this warp's 64 columns ----
      float s[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int kp = 0; kp < 2; ++kp) {
          const int key = nt * 8 + (lane & 7);
          const int c = 8 * warp + 4 * kp + (lane >> 3);
          uint32_t bq[4];
          ldmatrix_x4(bq, kvs + key * (kDim * 2) + ((c ^ (key & 7)) << 4));
          mma_16816(s[nt], qa[2 * kp], bq[0], bq[1]);
          mma_16816(s[nt], qa[2 * kp + 1], bq[2], bq[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int key = nt * 8 + 2 * q4;
        *reinterpret_cast<float2*>(&S.red[warp][g8][key]) = make_float2(s[nt][0], s[nt][1]);
        *reinterpret_cast<float2*>(&S.red[warp][g8 + 8][key]) = make_float2(s[nt][2], s[nt][3]);
      }
      __syncthreads();

      // ---- online softmax (16 threads per head) ----
      {
        float x0 = 0.f, x1 = 0.f;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
          const float2 v = *reinterpret_cast<const float2*>(&S.red[w][sh][2 * sj]);
          x0 += v.x;
          x1 += v.y;
        }
        x0 = ((vmask >> (2 * sj)) & 1u) ? x0 * p.scale_log2 : -INFINITY;
        x1 = ((vmask >> (2 * sj + 1)) & 1u) ? x1 * p.scale_log2 : -INFINITY;
        float bm = fmaxf(x0, x1);
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
        const float m_new = fmaxf(m_run, bm);
        const float base = (m_new == -INFINITY) ? 0.f : m_new;
        const float corr = exp2f(m_run - base);
        const float p0 = exp2f(x0 - base), p1 = exp2f(x1 - base);
        float ps = p0 + p1;
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l_run = l_run * corr + ps;
        m_run = m_new;
        *reinterpret_cast<uint32_t*>(&S.p[sh][2 * sj]) = pack_bf16x2(p0, p1);
        if (sj == 0) S.corr[sh] = corr;
      }
      __syncthreads();

      // ---- O = O * corr + P V over this warp's 64 columns ----
      const float c_lo = S.corr[g8], c_hi = S.corr[g8 + 8];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        o[nt][0] *= c_lo;
        o[nt][1] *= c_lo;
        o[nt][2] *= c_hi;
        o[nt][3] *= c_hi;
      }
      const uint32_t pbase = smem_u32(&S.p[0][0]);
#pragma unroll
      for (int kst = 0; kst < 2; ++kst) {
        uint32_t pa[4];
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kst * 16 + (lane >> 4) * 8;
        ldmatrix_x4(pa, pbase + row * (P_LD * 2) + col * 2);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int key = kst * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = 8 * warp + 2 * np + (lane >> 4);
          uint32_t vb[4];
          ldmatrix_x4_trans(vb, kvs + key * (kDim * 2) + ((c ^ (key & 7)) << 4));
          mma_16816(o[2 * np], pa, vb[0], vb[1]);
          mma_16816(o[2 * np + 1], pa, vb[2], vb[3]);
        }
      }
    }

    if (seg_end) {
      if (sj == 0) {
        S.mrun[sh] = m_run;
        S.lrun[sh] = l_run;
      }
      __syncthreads();
      const float m_lo = S.mrun[g8], l_lo = S.lrun[g8];
      const float m_hi = S.mrun[g8 + 8], l_hi = S.lrun[g8 + 8];
      const int64_t tb = t / p.m, tm = t - tb * p.m;
      if (seg_kb0 == 0 && kb == upt - 1) {
        const float f_lo = sink_factor(m_lo, l_lo, __ldg(p.sink + g8) * kLog2e);
        const float f_hi = sink_factor(m_hi, l_hi, __ldg(p.sink + g8 + 8) * kLog2e);
        __nv_bfloat16* ob = p.o + tb * p.o_sb + tm * p.o_sm;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int d = 64 * warp + 8 * nt + 2 * q4;
          *reinterpret_cast<uint32_t*>(ob + g8 * p.o_sh + d) =
              pack_bf16x2(o[nt][0] * f_lo, o[nt][1] * f_lo);
          *reinterpret_cast<uint32_t*>(ob + (g8 + 8) * p.o_sh + d) =
              pack_bf16x2(o[nt][2] * f_hi, o[nt][3] * f_hi);
        }
      } else {
        const int64_t slot = 2 * g + (t == t_first ? 0 : 1);
        float* pacc = p.part_acc + slot * kPartAccFloats;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int d = 64 * warp + 8 * nt + 2 * q4;
          *reinterpret_cast<float2*>(pacc + g8 * kDim + d) = make_float2(o[nt][0], o[nt][1]);
          *reinterpret_cast<float2*>(pacc + (g8 + 8) * kDim + d) = make_float2(o[nt][2], o[nt][3]);
        }
        if (tid < kHeads) {
          p.part_ml[slot * kPartMlFloats + tid] = S.mrun[tid];
          p.part_ml[slot * kPartMlFloats + kHeads + tid] = S.lrun[tid];
        }
      }
    }
  }
  cp_async_wait<0>();
}

}  // namespace mma_path

// ----------------------------------------------------------------------------
// LSE combine of split rows (shared by every variant).
// A row is split when the CTA that ends it ("owner") starts inside it.  Block
// (j, h) merges head h of the j-th split row: the fp32 partials of CTAs
// f..owner with the sink as the extra logit (reference.py:34-38); partial
// slots follow the rule in sa_common.cuh.  64 threads x 8 columns, all loads
// of a thread (maxima, sums and data of up to kCombineBatch partials) issued
// together: one memory round trip.  The blocks are small (64 threads, <= 128
// registers, no shared memory) so that, launched as programmatic dependents
// of the forward kernel, they become resident beside its CTAs and start the
// moment griddepcontrol.wait releases them (forward grid complete, stores
// visible).
// ----------------------------------------------------------------------------
constexpr int kMaxOwners = 512;  // >= the largest persistent grid (2 x SM count)

struct OwnerList {
  uint16_t cta[kMaxOwners];  // owner CTA of each split row, in CTA order
};

__host__ __device__ inline bool owns_split_row(int64_t g, int64_t U, int64_t G, int64_t upt) {
  const int64_t u0 = unit_begin(g, U, G), u1 = unit_begin(g + 1, U, G);
  if (u0 >= u1) return false;
  const int64_t ts = (u0 / upt) * upt;
  return u0 != ts && u1 >= ts + upt;
}

__global__ void __launch_bounds__(64, 8) sa_combine_kernel(const Params p,
                                                          const __grid_constant__ OwnerList owners) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t G = p.grid, U = p.units, upt = p.upt;
  const int64_t g = owners.cta[blockIdx.x];
  const int64_t u0 = unit_begin(g, U, G);
  const int64_t t = u0 / upt, ts = t * upt;
  const int64_t f = cta_of_unit(ts, U, G);
  const bool f_mid = unit_begin(f, U, G) < ts;
  const int np = static_cast<int>(g - f + 1);

  if (p.hg > 1) {  // blockIdx.z: the head group (Params::hg)
    merge_split_row(group_params(p, blockIdx.z), f, np, f_mid, t, blockIdx.y, threadIdx.x * 8);
  } else {
    merge_split_row(p, f, np, f_mid, t, blockIdx.y, threadIdx.x * 8);
  }
}

// Owner CTAs of the split rows (the combine kernel's blocks).
int split_rows(const Params& p, OwnerList* list) {
  int n = 0;
  for (int64_t g = 1; g < p.grid && n < kMaxOwners; ++g)
    if (owns_split_row(g, p.units, p.grid, p.upt)) list->cta[n++] = static_cast<uint16_t>(g);
  return n;
}

cudaError_t launch_combine(const Params& p, cudaStream_t st) {
#ifdef SA_NO_COMBINE  // development builds only: time the forward kernel alone
  return cudaSuccess;
#endif
  OwnerList owners;
  const int rows = split_rows(p, &owners);
  if (rows == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows), kHeads, static_cast<unsigned>(p.hg));
  cfg.blockDim = dim3(64, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sa_combine_kernel, p, owners);
}

int mma_unit_keys() { return mma_path::BN; }

int read_mma_index_faults(unsigned long long* out, bool reset) {
  return index_fault_io(sa_mma_index_faults, out, reset);
}

size_t mma_smem_bytes() { return sizeof(mma_path::Smem); }

cudaError_t launch_mma(const Params& p, cudaStream_t st) {
  const size_t smem = sizeof(mma_path::Smem);
  static PerDeviceOnce attr_once;
  cudaError_t e = once_per_device(attr_once, [&] {
    return cudaFuncSetAttribute(mma_path::sa_mma_fwd_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (e != cudaSuccess) return e;
  mma_path::sa_mma_fwd_kernel<<<p.grid, mma_path::NT, smem, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_combine(p, st);
}

}  // namespace sa
