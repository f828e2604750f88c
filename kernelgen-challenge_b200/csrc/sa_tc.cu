// sa_tc.cu — persistent gather-attend kernel on the sm_100a tensor path:
// tcgen05.mma with TMEM accumulators, KV rows gathered by cp.async into the
// 128-byte-swizzled operand layout, Q loaded by TMA.
//
// Algorithm: track-01/submission.py:276-347 (math of reference.py:24-40);
// masking of submission.py:313-322; sink in the denominator only
// (submission.py:340-345).  Work schedule and split/combine: sa_common.cuh.
//
// Per 64-key unit (64 KiB of gathered rows), swap-AB so that the 16 heads sit
// on the MMA's N dimension:
//   S^T[64 keys x 16 heads] = K[64 x 512] . Q^T[512 x 16]    (M=64,  N=16, 32 MMAs)
//   O^T[512 d x 16 heads]  += V^T[512 x 64] . P^T[64 x 16]    (M=128, N=16, 4x4 MMAs)
// K and V are the same shared-memory tile: read K-major for S^T and MN-major
// for O^T.  The tile is 8 slabs of [64 keys x 64 columns] in the 128-byte
// swizzle; Q is 8 slabs of [16 heads x 64 columns].
//
// Row gathers use cp.async from 128 threads: for random 1 KiB rows it moves
// more bytes per SM than TMA tile::gather4 (whose per-instruction issue cost
// caps a single producer warp near 2 TB/s on B200).
//
// Warp roles (320 threads, one CTA per SM):
//   warps 0..3   KV producer: indices -> 32 cp.async per thread per unit into a
//                3-deep ring of 64 KiB slots (full/empty mbarriers)
//   warp 8       TMEM owner and MMA issuer (one thread): S^T(i) into a double-buffered TMEM
//                tile, then O^T += V^T P^T for unit i-1 (so S(i) overlaps the
//                softmax of unit i-1)
//   warp 9       Q producer: one tiled TMA per 64 columns when a row starts
//   warps 4..7   softmax + epilogue; warp 4+q reads TMEM lane quarter q.
//                Thread = key: 16 scores per thread, no cross-thread reduction
//                in the common case.  The running max is only raised when a
//                score exceeds it by more than 2^8 (checked by one barrier
//                vote per unit); then the block max is reduced and O^T in
//                TMEM and the per-thread partial sums are rescaled.  The result
//                is exact for any threshold: P <= 2^8 is safe in bf16/fp32.
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error code
// in sa_tc_error (readable through sa_device_status) and stops issuing work.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "sa_tc.cuh"

namespace sa {

__device__ int sa_tc_error;  // nonzero after a bounded wait gave up

namespace tc_path {
using namespace tc;

constexpr int UK = 64;               // keys per unit
constexpr int NSLOT = 3;             // ring depth (units)
constexpr int SLOT_BYTES = UK * kDim * 2;  // 64 KiB
constexpr int SLAB_BYTES = UK * 128;       // [64 keys x 64 cols] = 8 KiB
constexpr int Q_BYTES = kHeads * kDim * 2; // 16 KiB
constexpr int P_BYTES = UK * kHeads * 2;   // 2 KiB
constexpr int NT = 320;  // 4 producer, 4 softmax, MMA, Q warps
constexpr float kRescaleThreshold = 8.0f;  // log2 domain
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kTmemS = 0;   // two S^T buffers: cols [0,16), [16,32)
constexpr uint32_t kTmemO = 32;  // O^T chunks: cols [32 + 16c, 48 + 16c)

struct __align__(1024) Smem {
  uint8_t ring[NSLOT][SLOT_BYTES];
  uint8_t q[Q_BYTES];
  uint8_t p[2][P_BYTES];
  uint32_t mask[NSLOT][2];  // validity: [0] keys 2l, [1] keys 2l+1 (bit l)
  float red_max[4][kHeads];
  float red_l[4][kHeads];
  uint64_t full[NSLOT], empty[NSLOT], q_full, q_empty, s_full[2], p_full[2];
  uint32_t tmem_base;
  int err;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + manual 1 KiB alignment

__device__ __forceinline__ void set_err(Smem& S, int code) {
  if (atomicCAS(&S.err, 0, code) == 0) atomicCAS(&sa_tc_error, 0, code);
}

// Bounded wait that also gives up at once when another warp recorded an error.
// After an error every role keeps walking its loop (so all threads reach the
// same named barriers) but issues no more TMA or MMA work.
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

  if (tid == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(smem_u32(&S.full[s]), 128 + 1);
      mbar_init(smem_u32(&S.empty[s]), 1);
    }
    mbar_init(smem_u32(&S.q_full), 1);
    mbar_init(smem_u32(&S.q_empty), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&S.s_full[b]), 1);
      mbar_init(smem_u32(&S.p_full[b]), 4);
    }
    S.err = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc<kTmemCols>(smem_u32(&S.tmem_base));
    tmem_relinquish();
  }
  if (warp == 9 && lane == 0) tma_prefetch_desc(&q_map);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp < 4) {
    // ------------------------------------------------------------ KV producer
    // 128 threads; thread pt copies 16-byte chunk c = pt & 63 of the 32 rows
    // with parity pt >> 6, so every warp-wide cp.async reads 512 contiguous
    // bytes of one row.  The rows land in the 128-byte-swizzled slab layout.
    const uint64_t pol = l2_policy_evict_first();
    const int pt = tid, c = pt & 63, par = pt >> 6, j = c >> 3, cc = c & 7;
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
        if (lane == 0) {
          S.mask[slot][0] = ma;
          S.mask[slot][1] = mb;
        }
      }
      const __nv_bfloat16* kvb = p.kv + cur_tb * p.kv_sb + c * 8;
      const uint32_t dst0 = smem_u32(S.ring[slot]) + j * SLAB_BYTES;
      const int32_t mine = par ? ib : ia;
#pragma unroll 8
      for (int k = 0; k < UK / 2; ++k) {
        const int r = par + 2 * k;
        const int32_t id = __shfl_sync(0xffffffffu, mine, k);
        const bool v = id >= 0 && (int64_t)id < p.kv_len;
        cp_async16_hint(dst0 + r * 128 + ((cc ^ (r & 7)) << 4),
                        kvb + (v ? (int64_t)id : 0) * p.kv_sn, v ? 16 : 0, pol);
      }
      // the slot's full barrier counts 128 hardware arrivals (one per thread,
      // when its copies land) plus the mask writer's release arrival
      cp_async_mbar_arrive_noinc(smem_u32(&S.full[slot]));
      if (warp == 0 && lane == 0) mbar_arrive(smem_u32(&S.full[slot]));
    }
    cp_async_wait<0>();
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(64, 16, false, false);
      constexpr uint32_t idO = idesc_bf16(128, 16, true, true);
      const uint32_t q_base = smem_u32(S.q);
      int64_t kb = kb_first;
      int seg = 0;
      bool seg_first = true;      // unit i is the first of its segment
      bool prev_seg_first = true; // unit i-1 was the first of its segment
      auto issue_pv = [&](int j, bool first) {
        if (!wait_or_err(S, S.p_full[j & 1], (j >> 1) & 1, 2)) return;
        tc_fence_after();
        const uint32_t slot_base = smem_u32(S.ring[j % NSLOT]);
        const uint32_t pb = smem_u32(S.p[j & 1]);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad =
                smem_desc(slot_base + 2 * c * SLAB_BYTES + kk * 2048, SLAB_BYTES, 1024,
                          kLayoutSw128);
            const uint64_t bd = smem_desc(pb + kk * 512, 256, 128, kLayoutNone);
            mma_f16_ss(tmem + kTmemO + 16 * c, ad, bd, idO, !(first && kk == 0));
          }
        mma_commit(smem_u32(&S.empty[j % NSLOT]));
      };
      for (int i = 0; i < n; ++i) {
        const bool seg_end = (i == n - 1) || kb == upt - 1;
        // at a row boundary finish the previous row first: its epilogue must
        // not wait for the next row's Q
        if (i > 0 && seg_first) issue_pv(i - 1, prev_seg_first);
        const int slot = i % NSLOT;
        bool ok = !seg_first || wait_or_err(S, S.q_full, seg & 1, 3);
        ok = ok && wait_or_err(S, S.full[slot], (i / NSLOT) & 1, 4);
        if (ok) {
          fence_proxy_async_smem();  // cp.async (generic proxy) writes -> MMA reads
          tc_fence_after();
          const uint32_t slot_base = smem_u32(S.ring[slot]);
#pragma unroll
          for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad =
                  smem_desc(slot_base + j * SLAB_BYTES + kk * 32, 16, 1024, kLayoutSw128);
              const uint64_t bd =
                  smem_desc(q_base + j * 2048 + kk * 32, 16, 1024, kLayoutSw128);
              mma_f16_ss(tmem + kTmemS + 16 * (i & 1), ad, bd, idS, (j | kk) != 0);
            }
          mma_commit(smem_u32(&S.s_full[i & 1]));
          if (seg_end) mma_commit(smem_u32(&S.q_empty));
        }
        if (i > 0 && !seg_first) issue_pv(i - 1, prev_seg_first);
        prev_seg_first = seg_first;
        seg_first = seg_end;
        if (seg_end) ++seg;
        kb = (kb + 1 == upt) ? 0 : kb + 1;
      }
      issue_pv(n - 1, prev_seg_first);
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ Q producer
    if (lane == 0) {
      for (int64_t t = t_first; t <= t_last; ++t) {
        const int s = static_cast<int>(t - t_first);
        if (s > 0 && !wait_or_err(S, S.q_empty, (s - 1) & 1, 5)) continue;
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
    // ------------------------------------------------- softmax + epilogue
    const int qd = warp - 4;            // TMEM lane quarter
    const int key = 16 * qd + lane;     // key of this thread (lane < 16)
    const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
    float m_run[kHeads], l_part[kHeads];
    int64_t t = t_first, kb = kb_first, seg_kb0 = kb_first;
    bool seg_first = true;
    for (int i = 0; i < n; ++i) {
      const bool seg_end = (i == n - 1) || kb == upt - 1;
      if (seg_first) {
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          m_run[h] = -INFINITY;
          l_part[h] = 0.f;
        }
        seg_kb0 = kb;
      }
      const int slot = i % NSLOT;
      wait_or_err(S, S.full[slot], (i / NSLOT) & 1, 6);
      wait_or_err(S, S.s_full[i & 1], (i >> 1) & 1, 7);
      tc_fence_after();
      float x[kHeads];
      tmem_ld16(tmem + lane_off + kTmemS + 16 * (i & 1), x);
      tmem_wait_ld();
      const uint32_t mw = S.mask[slot][lane & 1];
      const bool valid = lane < 16 && ((mw >> (key >> 1)) & 1u);
      bool over = false;
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        x[h] = valid ? x[h] * p.scale_log2 : -INFINITY;
        over |= x[h] > m_run[h] + kRescaleThreshold;
      }
      if (named_bar_or(1, 128, over)) {
        // raise the running max to the block max (rare after the first unit)
        float bm[kHeads];
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          float v = x[h];
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
          bm[h] = v;
        }
        if (lane == 0)
#pragma unroll
          for (int h = 0; h < kHeads; ++h) S.red_max[qd][h] = bm[h];
        named_bar(2, 128);
        float corr[kHeads];
        bool any_corr = false;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          const float b4 = fmaxf(fmaxf(S.red_max[0][h], S.red_max[1][h]),
                                 fmaxf(S.red_max[2][h], S.red_max[3][h]));
          const float m_new = fmaxf(m_run[h], b4);
          corr[h] = (m_new == m_run[h]) ? 1.f : exp2f(m_run[h] - m_new);
          any_corr |= corr[h] != 1.f;
          m_run[h] = m_new;
          l_part[h] *= corr[h];
        }
        if (!seg_first && any_corr) {
          // O^T holds units up to i-1 of this segment: wait for its last PV
          const int j = i - 1;
          wait_or_err(S, S.empty[j % NSLOT], (j / NSLOT) & 1, 8);
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[16];
            tmem_ld16(tmem + lane_off + kTmemO + 16 * c, v);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < kHeads; ++h) v[h] *= corr[h];
            tmem_st16(tmem + lane_off + kTmemO + 16 * c, v);
          }
          tmem_wait_st();
        }
      }
      // P^T for this thread's key: bf16 [key][head] in 8x16-byte core matrices
      float pr[kHeads];
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        const float base = (m_run[h] == -INFINITY) ? 0.f : m_run[h];
        pr[h] = exp2f(x[h] - base);
        l_part[h] += pr[h];
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
        uint8_t* pb = S.p[i & 1] + (key >> 3) * 256 + (key & 7) * 16;
        *reinterpret_cast<uint4*>(pb) = lo;
        *reinterpret_cast<uint4*>(pb + 128) = hi;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.p_full[i & 1]));

      if (seg_end) {
        // ---------------- epilogue of the segment ending at unit i ----------
        float lt[kHeads];
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          float v = l_part[h];
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
          lt[h] = v;
        }
        if (lane == 0)
#pragma unroll
          for (int h = 0; h < kHeads; ++h) S.red_l[qd][h] = lt[h];
        named_bar(2, 128);
#pragma unroll
        for (int h = 0; h < kHeads; ++h)
          lt[h] = (S.red_l[0][h] + S.red_l[1][h]) + (S.red_l[2][h] + S.red_l[3][h]);
        wait_or_err(S, S.empty[slot], (i / NSLOT) & 1, 9);  // PV(i) done
        tc_fence_after();
        const int64_t tb = t / p.m, tm = t - tb * p.m;
        const bool whole = (seg_kb0 == 0) && (kb == upt - 1);
        if (whole) {
          float f[kHeads];
#pragma unroll
          for (int h = 0; h < kHeads; ++h)
            f[h] = sink_factor(m_run[h], lt[h], __ldg(p.sink + h) * kLog2e);
          __nv_bfloat16* ob = p.o + tb * p.o_sb + tm * p.o_sm;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[16];
            tmem_ld16(tmem + lane_off + kTmemO + 16 * c, v);
            tmem_wait_ld();
            const int d = 128 * c + 32 * qd + lane;
#pragma unroll
            for (int h = 0; h < kHeads; ++h) ob[h * p.o_sh + d] = __float2bfloat16_rn(v[h] * f[h]);
          }
        } else {
          const int64_t pslot = 2 * g + (t == t_first ? 0 : 1);
          float* pacc = p.part_acc + pslot * kPartAccFloats;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[16];
            tmem_ld16(tmem + lane_off + kTmemO + 16 * c, v);
            tmem_wait_ld();
            const int d = 128 * c + 32 * qd + lane;
#pragma unroll
            for (int h = 0; h < kHeads; ++h) pacc[h * kDim + d] = v[h];
          }
          if (qd == 0 && lane == 0) {
#pragma unroll
            for (int h = 0; h < kHeads; ++h) {
              p.part_ml[pslot * kPartMlFloats + h] = m_run[h];
              p.part_ml[pslot * kPartMlFloats + kHeads + h] = lt[h];
            }
          }
        }
        tc_fence_before();
        named_bar(2, 128);  // O^T fully read before the next segment's first PV
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
  if (warp == 8) {
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

bool tc_available() { return true; }
int tc_unit_keys() { return tc_path::UK; }
int tc_ctas_per_sm() { return 1; }

// Conditions under which the Q tensor map can describe the inputs.
bool tc_supports(const Params& p) {
  if (p.m >= INT32_MAX || p.b >= INT32_MAX) return false;
  return (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0;
}

cudaError_t launch_tc(const Params& p, cudaStream_t st) {
  using namespace tc_path;
  auto enc = encoder();
  if (enc == nullptr) return cudaErrorNotSupported;
  CUtensorMap q_map;
  {
    cuuint64_t dims[4] = {(cuuint64_t)kDim, (cuuint64_t)kHeads, (cuuint64_t)p.m, (cuuint64_t)p.b};
    cuuint64_t strides[3] = {(cuuint64_t)p.q_sh * 2, (cuuint64_t)p.q_sm * 2,
                             (cuuint64_t)p.q_sb * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)kHeads, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&q_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<__nv_bfloat16*>(p.q), dims,
            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaFuncSetAttribute(sa_tc_fwd_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  sa_tc_fwd_kernel<<<p.grid, NT, kSmemBytes, st>>>(p, q_map);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_combine(p, st);
}

int read_tc_error(int* flags) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, sa_tc_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  *flags = v;
  return 0;
}

}  // namespace sa
