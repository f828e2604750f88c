// sa_tc.cu — persistent gather-attend kernel for sm_100a: tcgen05 tensor cores
// for the scores, warp MMAs for P.V, KV rows gathered by cp.async into the
// 128-byte-swizzled operand layout, Q loaded by TMA.
//
// Algorithm: track-01/submission.py:276-347 (math of reference.py:24-40);
// masking of submission.py:313-322; sink in the denominator only
// (submission.py:340-345).  Work schedule and split/combine: sa_common.cuh.
//
// Per 64-key unit (64 KiB of gathered rows):
//   S^T[64 keys x 16 heads] = K[64 x 512] . Q^T[512 x 16]
//       tcgen05.mma, M=64 (keys) N=16 (heads), accumulator in TMEM, split into
//       4 independent partial accumulators (8 MMAs each) so the MMAs pipeline.
//   O[16 heads x 512] += P[16 x 64] . V[64 x 512]
//       mma.sync m16n8k16 in the four softmax warps, O in registers (each warp
//       owns 128 columns), V read with ldmatrix.trans straight from the same
//       swizzled tile that the tensor core read as K.
// Why the split: a tcgen05.mma costs ~60 cycles of issue whatever M (64/128)
// and N (<= 128) are, so at N = 16 heads the 16 P.V MMAs per unit (M=128
// d-rows, N=16, K=16 keys) took as long as the 32 S MMAs and the single issuing
// thread bounded the pipeline; P.V as warp MMAs costs the softmax warps about
// 0.3 us per unit and runs concurrently with the next unit's S^T.
//
// Warp roles (256 threads, one CTA per SM; few enough threads that the
// softmax warps never spill: spill reloads queue behind the producer's
// outstanding copies in the load/store pipe and stall for microseconds):
//   warps 0..1   KV producer: 64 cp.async (16 B) per thread per unit into a
//                3-deep ring of 64 KiB slots; completion by hardware arrival
//                on the slot's full barrier
//   warp 2       TMEM owner; one thread issues S^T(i) into TMEM buffer i&1
//   warp 3       Q producer: one tiled TMA per 64 columns when a row starts
//   warps 4..7   softmax, P.V and epilogue; warp 4+q reads TMEM lane quarter
//                q (keys 16q..16q+15) and owns output columns [128q, 128q+128).
//                Thread = key for the softmax: no cross-thread reduction in the
//                common case.  The running max is only raised when a score
//                exceeds it by more than 2^8 (one barrier vote per unit); then
//                the block max is reduced and O and the partial sums are
//                rescaled.  Exact for any threshold: P <= 2^8 is safe in bf16.
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error code
// in sa_tc_error (readable through sa_device_status) and stops issuing work.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "sa_tc.cuh"

namespace sa {

__device__ int sa_tc_error;  // nonzero after a bounded wait gave up
__device__ unsigned long long sa_tc_index_faults;  // out-of-range indices seen


namespace tc_path {
using namespace tc;

constexpr int UK = 64;                      // keys per unit
constexpr int NSLOT = 3;                    // ring depth (units)
constexpr int SLOT_BYTES = UK * kDim * 2;   // 64 KiB
constexpr int SLAB_BYTES = UK * 128;        // [64 keys x 64 cols] = 8 KiB
constexpr int Q_BYTES = kHeads * kDim * 2;  // 16 KiB
constexpr int P_BYTES = UK * kHeads * 2;    // 2 KiB, P^T [key][head] bf16
constexpr int NT = 256;                     // 2 producer, MMA, Q, 4 softmax warps
constexpr float kRescaleThreshold = 8.0f;   // log2 domain
constexpr int kSAcc = 4;                    // independent S^T accumulators per unit
constexpr uint32_t kTmemCols = 128;         // S^T buffer b, partial a: cols 16*(4b + a)

struct __align__(1024) Smem {
  uint8_t ring[NSLOT][SLOT_BYTES];
  uint8_t q[Q_BYTES];
  uint8_t p[P_BYTES];
  uint32_t mask[NSLOT][2];  // validity: [0] keys 2l, [1] keys 2l+1 (bit l)
  float red_max[4][kHeads];
  // full: rows landed (128 cp.async arrivals + mask writer); empty: the four
  // softmax warps finished P.V on the slot; s_full: S^T(i) in TMEM; s_free:
  // the softmax warps read S^T out of TMEM buffer i&1
  uint64_t full[NSLOT], empty[NSLOT], q_full, q_empty, s_full[2], s_free[2];
  uint32_t tmem_base;
  int err;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + manual 1 KiB alignment

__device__ __forceinline__ void set_err(Smem& S, int code) {
  if (atomicCAS(&S.err, 0, code) == 0) atomicCAS(&sa_tc_error, 0, code);
}

// Bounded wait that also gives up at once when another warp recorded an error.
// After an error every role keeps walking its loop (so all threads reach the
// same named barriers) but issues no more copies or MMAs.
__device__ __forceinline__ bool wait_or_err(Smem& S, uint64_t& bar, uint32_t parity, int code) {
  const uint32_t b = smem_u32(&bar);
  if (*reinterpret_cast<volatile int*>(&S.err) != 0) return false;
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 1023u) == 1023u && *reinterpret_cast<volatile int*>(&S.err) != 0) return false;
  }
  set_err(S, code);
  return false;
}

// Byte offset of P^T[key][half] (8 heads = 16 B) in the P tile: rows of 32 B,
// halves swapped every 4 keys so ldmatrix reads of 8 keys hit 8 bank groups.
__device__ __forceinline__ uint32_t p_off(int key, int half) {
  return key * 32 + ((half ^ ((key >> 2) & 1)) << 4);
}

__global__ void __launch_bounds__(NT, 1)
    sa_tc_fwd_kernel(const Params p, const __grid_constant__ CUtensorMap q_map) {
  extern __shared__ uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t G = p.grid, g = blockIdx.x;
  const int64_t u0 = unit_begin(g, p.units, G), u1 = unit_begin(g + 1, p.units, G);
  const int n = static_cast<int>(u1 - u0);
  if (n <= 0) return;
  const int64_t upt = p.upt;
  const int64_t t_first = u0 / upt;
  const int64_t t_last = (u1 - 1) / upt;
  const int64_t kb_first = u0 - t_first * upt;
  // let the combine kernel of split rows launch now; it waits for this grid
  // to complete before reading any partial (griddepcontrol.wait)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (tid == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(smem_u32(&S.full[s]), 64 + 1);
      mbar_init(smem_u32(&S.empty[s]), 4);
    }
    mbar_init(smem_u32(&S.q_full), 1);
    mbar_init(smem_u32(&S.q_empty), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&S.s_full[b]), 1);
      mbar_init(smem_u32(&S.s_free[b]), 4);
    }
    S.err = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc<kTmemCols>(smem_u32(&S.tmem_base));
    tmem_relinquish();
  }
  if (warp == 3 && lane == 0) tma_prefetch_desc(&q_map);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp < 2) {
    // ------------------------------------------------------------ KV producer
    // 64 threads; thread c copies 16-byte chunk c of all 64 rows, so every
    // warp-wide cp.async reads 512 contiguous bytes of one row.  The rows land
    // in the 128-byte-swizzled slab layout.
    const uint64_t pol = l2_policy_evict_first();
    const int c = tid, j = c >> 3, cc = c & 7;
    int64_t t = t_first, kb = kb_first;
    int64_t tb = t / p.m, tm = t - tb * p.m;
    auto load_ids = [&](int64_t kb_, int64_t tb_, int64_t tm_, int32_t& a, int32_t& b) {
      const int64_t k0 = kb_ * UK + 2 * lane;
      const int32_t* base = p.idx + tb_ * p.i_sb + tm_ * p.i_sm;
      a = k0 < p.topk ? __ldg(base + k0 * p.i_sk) : -1;
      b = k0 + 1 < p.topk ? __ldg(base + (k0 + 1) * p.i_sk) : -1;
    };
    int32_t na, nb;
    load_ids(kb, tb, tm, na, nb);
    for (int i = 0; i < n; ++i) {
      const int32_t ia = na, ib = nb;
      const int64_t cur_tb = tb;
      // advance the cursor and prefetch the next unit's indices
      if (++kb == upt) {
        kb = 0;
        ++t;
        if (++tm == p.m) {
          tm = 0;
          ++tb;
        }
      }
      if (i + 1 < n) load_ids(kb, tb, tm, na, nb);

      const int slot = i % NSLOT;
      const bool ok = i < NSLOT || wait_or_err(S, S.empty[slot], ((i / NSLOT) - 1) & 1, 1);
      if (!__all_sync(0xffffffffu, ok)) continue;
      if (warp == 0) {
        const uint32_t ma = __ballot_sync(0xffffffffu, ia >= 0 && (int64_t)ia < p.kv_len);
        const uint32_t mb = __ballot_sync(0xffffffffu, ib >= 0 && (int64_t)ib < p.kv_len);
        const uint32_t fa = __ballot_sync(0xffffffffu, index_fault(ia, p.kv_len));
        const uint32_t fb = __ballot_sync(0xffffffffu, index_fault(ib, p.kv_len));
        if (lane == 0) {
          S.mask[slot][0] = ma;
          S.mask[slot][1] = mb;
          count_index_faults(&sa_tc_index_faults, __popc(fa) + __popc(fb));
        }
      }
      const __nv_bfloat16* kvb = p.kv + cur_tb * p.kv_sb + c * 8;
      const uint32_t dst0 = smem_u32(S.ring[slot]) + j * SLAB_BYTES;
#pragma unroll 8
      for (int k = 0; k < UK / 2; ++k) {
        const int32_t ida = __shfl_sync(0xffffffffu, ia, k);  // row 2k
        const int32_t idb = __shfl_sync(0xffffffffu, ib, k);  // row 2k+1
        const bool va = ida >= 0 && (int64_t)ida < p.kv_len;
        const bool vb = idb >= 0 && (int64_t)idb < p.kv_len;
        const int r = 2 * k;
        cp_async16_hint(dst0 + r * 128 + ((cc ^ (r & 7)) << 4),
                        kvb + (va ? (int64_t)ida : 0) * p.kv_sn, va ? 16 : 0, pol);
        cp_async16_hint(dst0 + (r + 1) * 128 + ((cc ^ ((r + 1) & 7)) << 4),
                        kvb + (vb ? (int64_t)idb : 0) * p.kv_sn, vb ? 16 : 0, pol);
      }
      // the slot's full barrier counts 64 hardware arrivals (one per thread,
      // when its copies land) plus the mask writer's release arrival
      cp_async_mbar_arrive_noinc(smem_u32(&S.full[slot]));
      if (warp == 0 && lane == 0) mbar_arrive(smem_u32(&S.full[slot]));
    }
    cp_async_wait<0>();
  } else if (warp == 2) {
    // ------------------------------------------------------------ S^T issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(64, 16, false, false);
      const uint32_t q_base = smem_u32(S.q);
      int64_t kb = kb_first;
      int seg = 0;
      bool seg_first = true;
      for (int i = 0; i < n; ++i) {
        const bool seg_end = (i == n - 1) || kb == upt - 1;
        const int slot = i % NSLOT;
        bool ok = !seg_first || wait_or_err(S, S.q_full, seg & 1, 3);
        ok = ok && wait_or_err(S, S.full[slot], (i / NSLOT) & 1, 4);
        // TMEM buffer i&1 was last read by the softmax of unit i-2
        ok = ok && (i < 2 || wait_or_err(S, S.s_free[i & 1], ((i - 2) >> 1) & 1, 5));
        if (ok) {
          fence_proxy_async_smem();  // cp.async (generic proxy) writes -> MMA reads
          tc_fence_after();
          const uint32_t slot_base = smem_u32(S.ring[slot]);
          const uint32_t d = tmem + 16 * kSAcc * (i & 1);
          // partial a accumulates slabs 2a and 2a+1; consecutive MMAs target
          // different partials so none waits for the previous one
#pragma unroll
          for (int j2 = 0; j2 < 8 / kSAcc; ++j2)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
#pragma unroll
              for (int a = 0; a < kSAcc; ++a) {
                const int sl = (8 / kSAcc) * a + j2;
                const uint64_t ad =
                    smem_desc(slot_base + sl * SLAB_BYTES + kk * 32, 16, 1024, kLayoutSw128);
                const uint64_t bd =
                    smem_desc(q_base + sl * 2048 + kk * 32, 16, 1024, kLayoutSw128);
                mma_f16_ss(d + 16 * a, ad, bd, idS, (j2 | kk) != 0);
              }
          mma_commit(smem_u32(&S.s_full[i & 1]));
          if (seg_end) mma_commit(smem_u32(&S.q_empty));
        }
        seg_first = seg_end;
        if (seg_end) ++seg;
        kb = (kb + 1 == upt) ? 0 : kb + 1;
      }
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------------------------------------ Q producer
    if (lane == 0) {
      for (int64_t t = t_first; t <= t_last; ++t) {
        const int s = static_cast<int>(t - t_first);
        if (s > 0 && !wait_or_err(S, S.q_empty, (s - 1) & 1, 6)) continue;
        const int64_t tb = t / p.m, tm = t - tb * p.m;
        mbar_arrive_expect_tx(smem_u32(&S.q_full), Q_BYTES);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tma_load_4d(smem_u32(S.q) + j * 2048, &q_map, 64 * j, 0, (int32_t)tm, (int32_t)tb,
                      smem_u32(&S.q_full));
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------- softmax + P.V + epilogue
    const int qd = warp - 4;         // TMEM lane quarter = key group = column quarter
    const int key = 16 * qd + lane;  // key of this thread for the softmax (lane < 16)
    const int g8 = lane >> 2, q4 = lane & 3;  // mma.sync fragment coordinates
    const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
    const uint32_t pbase = smem_u32(S.p);
    float m_run[kHeads];
    float o[16][4];  // O[heads g8, g8+8][128*qd + 8*nt + 2*q4 + {0,1}]
    float lacc[4];   // running sums: [0],[1] head g8, [2],[3] head g8+8 (P . 1)
    const uint32_t kOnes = 0x3F803F80u;  // bf16 pair (1, 1)
    int64_t t = t_first, kb = kb_first, seg_kb0 = kb_first;
    bool seg_first = true;
    for (int i = 0; i < n; ++i) {
      const bool seg_end = (i == n - 1) || kb == upt - 1;
      if (seg_first) {
#pragma unroll
        for (int h = 0; h < kHeads; ++h) m_run[h] = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
        lacc[0] = lacc[1] = lacc[2] = lacc[3] = 0.f;
        seg_kb0 = kb;
      }
      const int slot = i % NSLOT;
      wait_or_err(S, S.full[slot], (i / NSLOT) & 1, 7);
      wait_or_err(S, S.s_full[i & 1], (i >> 1) & 1, 8);
      tc_fence_after();
      float x[kHeads];
      {
        float y[kHeads];
        const uint32_t sb = tmem + lane_off + 16 * kSAcc * (i & 1);
        tmem_ld16(sb, x);
        tmem_ld16(sb + 16, y);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < kHeads; ++h) x[h] += y[h];
#pragma unroll 1
        for (int a = 2; a < kSAcc; ++a) {
          tmem_ld16(sb + 16 * a, y);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < kHeads; ++h) x[h] += y[h];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.s_free[i & 1]));

      const uint32_t mw = S.mask[slot][lane & 1];
      const bool valid = lane < 16 && ((mw >> (key >> 1)) & 1u);
      bool over = false;
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        x[h] = valid ? x[h] * p.scale_log2 : -INFINITY;
        over |= x[h] > m_run[h] + kRescaleThreshold;
      }
      // The vote barrier also orders this unit's P^T writes after every
      // warp's P.V of the previous unit (single P tile).
      if (named_bar_or(1, 128, over)) {
        // raise the running max to the block max (rare after a row's first unit)
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          float v = x[h];
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
          if (lane == 0) S.red_max[qd][h] = v;
        }
        named_bar(2, 128);
        float c_lo = 1.f, c_hi = 1.f;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          const float b4 = fmaxf(fmaxf(S.red_max[0][h], S.red_max[1][h]),
                                 fmaxf(S.red_max[2][h], S.red_max[3][h]));
          const float m_new = fmaxf(m_run[h], b4);
          const float corr = (m_new == m_run[h]) ? 1.f : exp2f(m_run[h] - m_new);
          m_run[h] = m_new;
          if (h == g8) c_lo = corr;
          if (h == g8 + 8) c_hi = corr;
        }
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          o[nt][0] *= c_lo;
          o[nt][1] *= c_lo;
          o[nt][2] *= c_hi;
          o[nt][3] *= c_hi;
        }
        lacc[0] *= c_lo;
        lacc[1] *= c_lo;
        lacc[2] *= c_hi;
        lacc[3] *= c_hi;
      }
      // P^T row of this thread's key (bf16)
      float pr[kHeads];
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        const float base = (m_run[h] == -INFINITY) ? 0.f : m_run[h];
        pr[h] = exp2f(x[h] - base);
      }
      if (lane < 16) {
        uint4 lo, hi;
        lo.x = pack_bf16x2(pr[0], pr[1]);
        lo.y = pack_bf16x2(pr[2], pr[3]);
        lo.z = pack_bf16x2(pr[4], pr[5]);
        lo.w = pack_bf16x2(pr[6], pr[7]);
        hi.x = pack_bf16x2(pr[8], pr[9]);
        hi.y = pack_bf16x2(pr[10], pr[11]);
        hi.z = pack_bf16x2(pr[12], pr[13]);
        hi.w = pack_bf16x2(pr[14], pr[15]);
        *reinterpret_cast<uint4*>(S.p + p_off(key, 0)) = lo;
        *reinterpret_cast<uint4*>(S.p + p_off(key, 1)) = hi;
      }
      named_bar(3, 128);  // P^T of all 64 keys written

      // O[16 x 128 cols of this warp] += P[16 x 64] . V[64 x 128]
      const uint32_t slot_base = smem_u32(S.ring[slot]);
#pragma unroll
      for (int kst = 0; kst < 4; ++kst) {
        uint32_t pa[4];
        {
          const int mtx = lane >> 3;
          const int kr = kst * 16 + (mtx >> 1) * 8 + (lane & 7);
          ldmatrix_x4_trans(pa, pbase + p_off(kr, mtx & 1));
        }
        mma_16816(lacc, pa, kOnes, kOnes);  // row sums of the bf16 P actually used
        const int kr = kst * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          const int slab = 2 * qd + (np >> 2);
          const int ch = ((np & 3) << 1) + (lane >> 4);
          uint32_t vb[4];
          ldmatrix_x4_trans(vb, slot_base + slab * SLAB_BYTES + kr * 128 + ((ch ^ (kr & 7)) << 4));
          mma_16816(o[2 * np], pa, vb[0], vb[1]);
          mma_16816(o[2 * np + 1], pa, vb[2], vb[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.empty[slot]));  // slot free for the producer

      if (seg_end) {
        // ---------------- epilogue of the segment ending at unit i ----------
        float m_lo = 0.f, m_hi = 0.f;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          if (h == g8) m_lo = m_run[h];
          if (h == g8 + 8) m_hi = m_run[h];
        }
        const float l_lo = lacc[0], l_hi = lacc[2];
        const int64_t tb = t / p.m, tm = t - tb * p.m;
        if (seg_kb0 == 0 && kb == upt - 1) {
          const float f_lo = sink_factor(m_lo, l_lo, __ldg(p.sink + g8) * kLog2e);
          const float f_hi = sink_factor(m_hi, l_hi, __ldg(p.sink + g8 + 8) * kLog2e);
          __nv_bfloat16* ob = p.o + tb * p.o_sb + tm * p.o_sm;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt) {
            const int d = 128 * qd + 8 * nt + 2 * q4;
            *reinterpret_cast<uint32_t*>(ob + g8 * p.o_sh + d) =
                pack_bf16x2(o[nt][0] * f_lo, o[nt][1] * f_lo);
            *reinterpret_cast<uint32_t*>(ob + (g8 + 8) * p.o_sh + d) =
                pack_bf16x2(o[nt][2] * f_hi, o[nt][3] * f_hi);
          }
        } else {
          const int64_t pslot = 2 * g + (t == t_first ? 0 : 1);
          float* pacc = p.part_acc + pslot * kPartAccFloats;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt) {
            const int d = 128 * qd + 8 * nt + 2 * q4;
            *reinterpret_cast<float2*>(pacc + g8 * kDim + d) = make_float2(o[nt][0], o[nt][1]);
            *reinterpret_cast<float2*>(pacc + (g8 + 8) * kDim + d) =
                make_float2(o[nt][2], o[nt][3]);
          }
          if (qd == 0 && q4 == 0) {
            p.part_ml[pslot * kPartMlFloats + g8] = m_lo;
            p.part_ml[pslot * kPartMlFloats + g8 + 8] = m_hi;
            p.part_ml[pslot * kPartMlFloats + kHeads + g8] = l_lo;
            p.part_ml[pslot * kPartMlFloats + kHeads + g8 + 8] = l_hi;
          }
        }
      }
      seg_first = seg_end;
      if (++kb == upt) {
        kb = 0;
        ++t;
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc<kTmemCols>(tmem);
  }
}

}  // namespace tc_path

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return encoder(); }

bool tc_available() { return true; }
int tc_unit_keys() { return tc_path::UK; }
int tc_ctas_per_sm() { return 1; }

// Conditions under which the Q tensor map can describe the inputs.
bool tc_supports(const Params& p) {
  if (p.m >= INT32_MAX || p.b >= INT32_MAX) return false;
  return (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0;
}

// 4-D tensor map of q [b, m, 16, 512] (any row strides) with 64 x 16 boxes
// in the 128-byte swizzle; shared by the kernels that load Q with TMA.
cudaError_t encode_q_map(const Params& p, CUtensorMap* q_map) {
  // the last map built by this thread, reused while q's address and layout
  // are unchanged (the common case of a serving loop with fixed buffers)
  struct Cached {
    const void* q = nullptr;
    int64_t m = 0, b = 0, sh = 0, sm = 0, sb = 0, heads = 0;
    CUtensorMap map;
  };
  thread_local Cached cache;
  const int64_t heads = (int64_t)kHeads * (p.hg > 1 ? p.hg : 1);  // every head group's
  if (cache.q == p.q && cache.m == p.m && cache.b == p.b && cache.sh == p.q_sh &&
      cache.sm == p.q_sm && cache.sb == p.q_sb && cache.heads == heads) {
    *q_map = cache.map;
    return cudaSuccess;
  }
  auto enc = encoder();
  if (enc == nullptr) return cudaErrorNotSupported;
  cuuint64_t dims[4] = {(cuuint64_t)kDim, (cuuint64_t)heads, (cuuint64_t)p.m, (cuuint64_t)p.b};
  cuuint64_t strides[3] = {(cuuint64_t)p.q_sh * 2, (cuuint64_t)p.q_sm * 2, (cuuint64_t)p.q_sb * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)kHeads, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  if (enc(q_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<__nv_bfloat16*>(p.q), dims,
          strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  cache.q = p.q;
  cache.m = p.m;
  cache.b = p.b;
  cache.sh = p.q_sh;
  cache.sm = p.q_sm;
  cache.sb = p.q_sb;
  cache.heads = heads;
  cache.map = *q_map;
  return cudaSuccess;
}

cudaError_t launch_tc(const Params& p, cudaStream_t st) {
  using namespace tc_path;
  CUtensorMap q_map;
  {
    const cudaError_t eq = encode_q_map(p, &q_map);
    if (eq != cudaSuccess) return eq;
  }
  static PerDeviceOnce attr_once;
  cudaError_t e = once_per_device(attr_once, [] {
    return cudaFuncSetAttribute(sa_tc_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  sa_tc_fwd_kernel<<<p.grid, NT, kSmemBytes, st>>>(p, q_map);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_combine(p, st);
}


int read_tc_index_faults(unsigned long long* out, bool reset) {
  return index_fault_io(sa_tc_index_faults, out, reset);
}

int read_tc_error(int* flags) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, sa_tc_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  *flags = v;
  return 0;
}

int reset_tc_error() {
  const int zero = 0;
  return (int)cudaMemcpyToSymbol(sa_tc_error, &zero, sizeof(int));
}

}  // namespace sa
