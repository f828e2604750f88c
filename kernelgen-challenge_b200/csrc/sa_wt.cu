// sa_wt.cu — warp-specialized persistent gather-attend kernel for sm_100a
// with the output accumulator in tensor memory: S = Q.K^T on warp MMAs
// (mma.sync m16n8k16, Q fragments in registers), O += P.V on tcgen05.mma
// with O in TMEM, issued by one thread and running while the consumer warps
// go on with the next unit's scores.
//
// Algorithm: track-01/submission.py:276-347 (math of reference.py:24-40);
// masking of submission.py:313-322; sink in the denominator only
// (submission.py:340-345).  Work schedule, split rows and their merges:
// sa_common.cuh, as in sa_ws.cu, whose producer this kernel repeats.
//
// Why split the products this way: with 16 heads, S^T on tcgen05 would put
// the heads on N = 16 and the 64 keys of a unit on M = 64: 32 instructions of
// ~60 cycles per unit from one thread, slower than four warps of mma.sync.
// P.V is the other way round: O^T [512 columns x 16 heads] = V^T . P^T puts
// the columns on M = 128, so a unit is 16 instructions (4 column blocks x 4
// key steps of 16), ~1000 tensor cycles that overlap the warps' own work, and
// the fp32 O (32 KiB per row) lives in 64 TMEM columns instead of 64
// registers per consumer thread.
//
// Operands of the P.V MMAs (kind::f16, bf16 x bf16 -> fp32, M = 128, N = 16,
// K = 16):
//   A = V^T, MN-major, 128-byte swizzle, straight from the ring slot: a slab
//       holds 64 keys x 64 columns, key r's 128-byte row with its 16-byte
//       chunks XOR-swizzled by r & 7, which is the MN-major swizzle atom
//       (64 columns x 8 keys).  LBO = 8 KiB (the next 64 columns: the next
//       slab), SBO = 1 KiB (the next 8 keys).
//   B = P^T, K-major, 128-byte swizzle: the P tile [16 heads][64 keys] bf16,
//       one 128-byte row per head, chunks swizzled by head & 7; SBO = 1 KiB.
//   D: column block j (columns 128j .. 128j+127) in TMEM lanes 0..127 (lane =
//       column), TMEM columns 16j .. 16j+15 (one per head).
//
// Per unit (consumer warp c = 0..3, keys 16c..16c+15 of S):
//   wait full -> S (64 MMAs) -> release the slot's S share -> vote on the
//   running max (rescale: wait for the MMAs in flight, then scale O in TMEM,
//   rare after a row's first unit) -> wait until the P buffer's previous MMAs
//   are done -> P (bf16) to shared memory, row sums in fp32 registers ->
//   barrier -> thread 0 issues the 16 MMAs and commits them to the slot's
//   empty barrier (V read) and to the P buffer's barrier.
// Segment end: wait for the segment's MMAs, read O from TMEM (each warp its
// 32 lanes, all 16 heads of a column per thread), normalise with the sink,
// store o (or the fp32 partial of a split row).
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error code
// in sa_wt_error (readable through sa_device_status as 400 + code), keeps
// walking its loops without issuing copies, waits for its MMAs and its TMA in
// flight (bounded) and frees its tensor memory before it exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "sa_tc.cuh"

namespace sa {

__device__ int sa_wt_error;                        // nonzero after a bounded wait gave up
__device__ unsigned long long sa_wt_index_faults;  // out-of-range indices seen

namespace wt_path {
using namespace tc;

constexpr int UK = 64;                      // keys per unit
constexpr int NSLOT = 3;                    // ring depth (units)
constexpr int SLOT_BYTES = UK * kDim * 2;   // 64 KiB
constexpr int SLAB_BYTES = UK * 128;        // [64 keys x 64 cols] = 8 KiB
constexpr int Q_BYTES = kHeads * kDim * 2;  // 16 KiB
constexpr int P_BYTES = kHeads * UK * 2;    // 2 KiB, P [head][key] bf16
constexpr int NCW = 4;                      // consumer warps
constexpr int NCT = NCW * 32;
constexpr int NT = 4 * 32 + NCT;            // 256
constexpr uint32_t kTmemCols = 64;          // 4 column blocks x 16 heads, fp32
constexpr float kRescaleThreshold = 8.0f;   // log2 domain

struct __align__(1024) Smem {
  uint8_t ring[NSLOT][SLOT_BYTES];
  uint8_t q[Q_BYTES];
  uint8_t p[2][P_BYTES];    // double-buffered: unit i writes p[i & 1]
  uint32_t mask[NSLOT][2];  // validity: [0] keys 2l, [1] keys 2l+1 (bit l)
  float red_max[NCW][kHeads];
  float red_sum[NCW][kHeads];
  float m_row[kHeads];  // running max per head (log2 domain), all heads
  float scl[kHeads];    // O rescale factors of the current vote
  // full: rows landed (128 cp.async arrivals + mask writer); empty: the four
  // consumer warps' S reads + the commit of the unit's P.V MMAs (V reads);
  // pv_done[b]: the MMAs that read P buffer b completed; q_full: next Q tile
  uint64_t full[NSLOT], empty[NSLOT], pv_done[2], q_full;
  uint32_t tmem;  // TMEM base address of O
  int err;
  uint32_t spin;  // polls before a wait gives up
  int n_merge;
  int64_t merge_row[2];
  int n_units;  // row schedule: units of this CTA
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + manual 1 KiB alignment
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ void set_err(Smem& S, int code) {
  if (atomicCAS(&S.err, 0, code) == 0) atomicCAS(&sa_wt_error, 0, code);
}

// Bounded wait that also gives up at once when another warp recorded an error.
__device__ __forceinline__ bool wait_or_err(Smem& S, uint64_t& bar, uint32_t parity, int code) {
  const uint32_t b = smem_u32(&bar);
  if (*reinterpret_cast<volatile int*>(&S.err) != 0) return false;
  for (uint32_t i = 0; i < S.spin; ++i) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 1023u) == 1023u && *reinterpret_cast<volatile int*>(&S.err) != 0) return false;
  }
  set_err(S, code);
  return false;
}

__device__ __forceinline__ uint32_t p_chunk(int h, int ch) {
  return h * 128 + ((ch ^ (h & 7)) << 4);
}

// TMEM address of lane `lane0`, column `col`.
__device__ __forceinline__ uint32_t tmem_at(uint32_t base, int lane0, int col) {
  return base + (static_cast<uint32_t>(lane0) << 16) + static_cast<uint32_t>(col);
}

// The 16 MMAs of one unit: O^T[128j + m][h] (+)= sum_k V[k][128j + m] P[h][k].
__device__ __forceinline__ void issue_pv(uint32_t tmem, uint32_t slot_base, uint32_t p_base,
                                         bool accumulate) {
  constexpr uint32_t idesc = idesc_bf16(128, 16, /*a_mn=*/true, /*b_mn=*/false);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint64_t bd = smem_desc(p_base + kk * 32, 16, 1024, kLayoutSw128);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint64_t ad =
          smem_desc(slot_base + 2 * j * SLAB_BYTES + kk * 2048, 8192, 1024, kLayoutSw128);
      mma_f16_ss(tmem + 16 * j, ad, bd, idesc, accumulate || kk != 0);
    }
  }
}

// One column block of O: 16 heads of column 128j + 32c + lane (this thread).
__device__ __forceinline__ void tmem_block(uint32_t tmem, int c, int j, float (&v)[16]) {
  tmem_ld16(tmem_at(tmem, 32 * c, 16 * j), v);
}

// kLse: also write the row log-sum-exp (training forward).  kRows: the row
// schedule of sa_common.cuh instead of contiguous unit ranges.
template <bool kLse, bool kRows>
__global__ void __launch_bounds__(NT, 1)
    sa_wt_fwd_kernel(const Params p, const __grid_constant__ CUtensorMap q_map) {
  extern __shared__ uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t G = p.grid, g = blockIdx.x;
  const int64_t R = p.b * p.m;
  int64_t u0 = 0, u1 = 0;
  if constexpr (kRows) {
    if (g >= R) return;  // (the host keeps R >= 2G)
  } else {
    u0 = unit_begin(g, p.units, G);
    u1 = unit_begin(g + 1, p.units, G);
    if (u1 <= u0) return;
  }
  int n = static_cast<int>(u1 - u0);  // units of this CTA (row schedule: below)
  const int64_t upt = p.upt;
  const int64_t t_first = kRows ? snake_row(0, g, G, R) : u0 / upt;
  const int64_t t_last = (u1 - 1) / upt;  // (unit ranges only)
  const int64_t kb_first = kRows ? 0 : u0 - t_first * upt;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (tid == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(smem_u32(&S.full[s]), 128 + 1);
      mbar_init(smem_u32(&S.empty[s]), NCW + 1);
    }
    mbar_init(smem_u32(&S.pv_done[0]), 1);
    mbar_init(smem_u32(&S.pv_done[1]), 1);
    mbar_init(smem_u32(&S.q_full), 1);
    S.err = 0;
    S.spin = p.spin != 0u ? p.spin : kSpinLimit;
    S.n_merge = 0;
    S.n_units = 0;
    fence_mbar_init();
  }
  if (warp == 4) {  // the first consumer warp owns the tensor memory
    tmem_alloc<kTmemCols>(smem_u32(&S.tmem));
    tmem_relinquish();
    if (lane == 0) tma_prefetch_desc(&q_map);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (kRows) {
    __syncthreads();  // (S.n_units initialised)
    int part = 0;
    for (int64_t k = tid;; k += NT) {
      const int64_t r = snake_row(k, g, G, R);
      if (r < 0) break;
      part += static_cast<int>(units_of_row(p, r));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    if (lane == 0 && part != 0) atomicAdd(&S.n_units, part);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (kRows) n = S.n_units;
  const uint32_t tmem = S.tmem;

  if (warp < 4) {
    // ------------------------------------------------------------ KV producer
    // As in sa_ws.cu: 128 threads; thread pt copies 16-byte chunk c = pt & 63
    // of the 32 rows of parity pt >> 6 (one warp-wide cp.async reads 512
    // contiguous bytes of one row) into the 128-byte-swizzled slab layout.
    const uint64_t pol = l2_policy_kv(p.kv_policy);
    const int c = tid & 63, par = tid >> 6, j = c >> 3, cc = c & 7;
    int64_t t = t_first, kb = kb_first;
    int64_t tb = t / p.m, tm = t - tb * p.m;
    int64_t sk = 0, nu_t = upt, nu_n = 0;
    if constexpr (kRows) {
      nu_t = units_of_row(p, t);
      nu_n = units_of_row(p, snake_row(1, g, G, R));
    }
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
      if (++kb == nu_t) {
        kb = 0;
        if constexpr (kRows) {
          t = snake_row(++sk, g, G, R);
          tb = t / p.m;
          tm = t - tb * p.m;
          nu_t = nu_n;
          nu_n = units_of_row(p, snake_row(sk + 1, g, G, R));
        } else {
          ++t;
          if (++tm == p.m) {
            tm = 0;
            ++tb;
          }
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
          count_index_faults(&sa_wt_index_faults, __popc(fa) + __popc(fb));
        }
      }
      const __nv_bfloat16* kvb = p.kv + cur_tb * p.kv_sb + c * 8;
      const uint32_t dst0 = smem_u32(S.ring[slot]) + j * SLAB_BYTES;
      const int32_t mine = par ? ib : ia;  // warp-uniform parity
#pragma unroll 8
      for (int k = 0; k < UK / 2; ++k) {
        const int32_t id = __shfl_sync(0xffffffffu, mine, k);  // row 2k + par
        const bool v = id >= 0 && (int64_t)id < p.kv_len;
        const int r = 2 * k + par;
        cp_async16_hint(dst0 + r * 128 + ((cc ^ (r & 7)) << 4),
                        kvb + (v ? (int64_t)id : 0) * p.kv_sn, v ? 16 : 0, pol);
      }
      cp_async_mbar_arrive_noinc(smem_u32(&S.full[slot]));
      // (failure-path test: the first slot's release is withheld)
      if (warp == 0 && lane == 0 && !(p.test_stall && i == 0)) mbar_arrive(smem_u32(&S.full[slot]));
    }
    cp_async_wait<0>();
  } else {
    // ------------------------------------------------------------ consumers
    const int c = warp - 4;                   // 0..3
    const int tt = tid - 128;                 // consumer thread 0..127
    const int g8 = lane >> 2, q4 = lane & 3;  // mma fragment coordinates
    const uint32_t qbase = smem_u32(S.q);
    uint32_t qf[32][4];                        // Q A-fragments, 32 k-steps of 16 columns
    float m_lo = -INFINITY, m_hi = -INFINITY;  // running max, heads g8 / g8+8 (log2)
    float l_lo = 0.f, l_hi = 0.f;              // this thread's share of the row sums
    int q_issued = 0;
    auto issue_q = [&](int64_t row) {
      if (*reinterpret_cast<volatile int*>(&S.err) != 0) return;
      ++q_issued;
      const int64_t qb = row / p.m, qm = row - qb * p.m;
      fence_proxy_async_smem();  // the Q fragment reads above precede the TMA refill
      mbar_arrive_expect_tx(smem_u32(&S.q_full), Q_BYTES);
#pragma unroll
      for (int jq = 0; jq < 8; ++jq)
        tma_load_4d(qbase + jq * 2048, &q_map, 64 * jq, 0, (int32_t)qm, (int32_t)qb,
                    smem_u32(&S.q_full));
    };
    int64_t t = t_first, kb = kb_first, seg_kb0 = kb_first;
    if (tt == 0) issue_q(t_first);
    int64_t sk = 0, nu_t = upt, nu_n = 0;
    if constexpr (kRows) {
      nu_t = units_of_row(p, t);
      nu_n = units_of_row(p, snake_row(1, g, G, R));
    }
    int seg = 0;
    bool seg_first = true;
    for (int i = 0; i < n; ++i) {
      const bool seg_end = (i == n - 1) || kb == nu_t - 1;
      const bool unit0 = seg_first;  // the segment's first unit: O is written, not added
      if (seg_first) {
        m_lo = m_hi = -INFINITY;
        l_lo = l_hi = 0.f;
        seg_kb0 = kb;
        wait_or_err(S, S.q_full, seg & 1, 7);
        {
          const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int ks = 0; ks < 32; ++ks) {
            const int ch = (ks & 3) * 2 + (lane >> 4);
            ldmatrix_x4(qf[ks], qbase + (ks >> 2) * 2048 + row * 128 + ((ch ^ (row & 7)) << 4));
          }
        }
        named_bar(4, NCT);
        if constexpr (kRows) {
          const int64_t tn = snake_row(sk + 1, g, G, R);
          if (tt == 0 && tn >= 0) issue_q(tn);
        } else if (tt == 0 && t < t_last) {
          issue_q(t + 1);
        }
      }
      const int slot = i % NSLOT;
      wait_or_err(S, S.full[slot], (i / NSLOT) & 1, 8);
      const uint32_t sb = smem_u32(S.ring[slot]);

      // ---- S for keys 16c + 8nt + {0..7}: 2 n-tiles x 32 k-steps, 2-way split
      float sa[2][2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int z = 0; z < 2; ++z) sa[nt][z][0] = sa[nt][z][1] = sa[nt][z][2] = sa[nt][z][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < 16; ++kp) {
        const int slab = kp >> 1, c0 = (kp & 1) * 4;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int key = 16 * c + 8 * nt + (lane & 7);
          uint32_t kf[4];
          ldmatrix_x4(kf, sb + slab * SLAB_BYTES + key * 128 + (((c0 + (lane >> 3)) ^ (key & 7)) << 4));
          mma_16816(sa[nt][0], qf[2 * kp], kf[0], kf[1]);
          mma_16816(sa[nt][1], qf[2 * kp + 1], kf[2], kf[3]);
        }
      }
      // this warp is done reading K from the slot; the P.V MMAs still read V
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.empty[slot]));

      const uint32_t mw0 = S.mask[slot][0], mw1 = S.mask[slot][1];
      float x[2][4];
      bool over = false;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int l = 8 * c + 4 * nt + q4;
        const bool v0 = (mw0 >> l) & 1u, v1 = (mw1 >> l) & 1u;
        x[nt][0] = v0 ? (sa[nt][0][0] + sa[nt][1][0]) * p.scale_log2 : -INFINITY;
        x[nt][1] = v1 ? (sa[nt][0][1] + sa[nt][1][1]) * p.scale_log2 : -INFINITY;
        x[nt][2] = v0 ? (sa[nt][0][2] + sa[nt][1][2]) * p.scale_log2 : -INFINITY;
        x[nt][3] = v1 ? (sa[nt][0][3] + sa[nt][1][3]) * p.scale_log2 : -INFINITY;
        over |= fmaxf(x[nt][0], x[nt][1]) > m_lo + kRescaleThreshold;
        over |= fmaxf(x[nt][2], x[nt][3]) > m_hi + kRescaleThreshold;
      }
      // The vote barrier also orders this unit's uses of S.red_max / S.scl
      // after the previous unit's.
      if (named_bar_or(1, NCT, over)) {
        float b_lo = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
        float b_hi = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
          b_lo = fmaxf(b_lo, __shfl_xor_sync(0xffffffffu, b_lo, off));
          b_hi = fmaxf(b_hi, __shfl_xor_sync(0xffffffffu, b_hi, off));
        }
        if (q4 == 0) {
          S.red_max[c][g8] = b_lo;
          S.red_max[c][g8 + 8] = b_hi;
        }
        named_bar(2, NCT);
        float n_lo = m_lo, n_hi = m_hi;
#pragma unroll
        for (int w = 0; w < NCW; ++w) {
          n_lo = fmaxf(n_lo, S.red_max[w][g8]);
          n_hi = fmaxf(n_hi, S.red_max[w][g8 + 8]);
        }
        const float c_lo = (n_lo == m_lo) ? 1.f : exp2f(m_lo - n_lo);
        const float c_hi = (n_hi == m_hi) ? 1.f : exp2f(m_hi - n_hi);
        m_lo = n_lo;
        m_hi = n_hi;
        l_lo *= c_lo;
        l_hi *= c_hi;
        if (c == 0 && q4 == 0) {
          S.m_row[g8] = m_lo;
          S.m_row[g8 + 8] = m_hi;
          S.scl[g8] = c_lo;
          S.scl[g8 + 8] = c_hi;
        }
        if (!unit0) {
          // O in TMEM holds earlier units: once their MMAs are done, scale
          // each head's column of every block (this thread: one O column)
          wait_or_err(S, S.pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1, 10);
          named_bar(2, NCT);  // (S.scl written)
          tc_fence_after();
#pragma unroll 1
          for (int jb = 0; jb < 4; ++jb) {
            float v[16];
            tmem_block(tmem, c, jb, v);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < 16; ++h) v[h] *= S.scl[h];
            tmem_st16(tmem_at(tmem, 32 * c, 16 * jb), v);
          }
          tmem_wait_st();
          tc_fence_before();
        }
      }
      // ---- P (bf16) into buffer i & 1, once the MMAs of unit i - 2 read it
      const int pbuf = i & 1;
      if (i >= 2) wait_or_err(S, S.pv_done[pbuf], ((i - 2) >> 1) & 1, 11);
      {
        const float base_lo = (m_lo == -INFINITY) ? 0.f : m_lo;
        const float base_hi = (m_hi == -INFINITY) ? 0.f : m_hi;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int ch = 2 * c + nt;  // keys 8ch..8ch+7
          const float p0 = exp2f(x[nt][0] - base_lo), p1 = exp2f(x[nt][1] - base_lo);
          const float p2 = exp2f(x[nt][2] - base_hi), p3 = exp2f(x[nt][3] - base_hi);
          l_lo += p0 + p1;
          l_hi += p2 + p3;
          *reinterpret_cast<uint32_t*>(S.p[pbuf] + p_chunk(g8, ch) + 4 * q4) = pack_bf16x2(p0, p1);
          *reinterpret_cast<uint32_t*>(S.p[pbuf] + p_chunk(g8 + 8, ch) + 4 * q4) =
              pack_bf16x2(p2, p3);
        }
      }
      fence_proxy_async_smem();  // P (generic stores) -> the MMAs' reads
      tc_fence_before();
      named_bar(3, NCT);  // P of all 64 keys written; any O rescale done
      if (tt == 0) {
        // V landed through cp.async (generic proxy): make it visible to the
        // MMAs' async-proxy reads, then issue the unit's 16 MMAs
        fence_proxy_async_smem();
        tc_fence_after();
        issue_pv(tmem, sb, smem_u32(S.p[pbuf]), !unit0);
        mma_commit(smem_u32(&S.empty[slot]));  // V reads done: the slot's last arrival
        mma_commit(smem_u32(&S.pv_done[pbuf]));
      }

      if (seg_end) {
        // ---------------- epilogue of the segment ending at unit i ----------
        const int64_t tb = t / p.m, tm = t - tb * p.m;
        // row sums of all heads: over the lanes of a fragment row, the warps
        float s_lo = l_lo, s_hi = l_hi;
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
          s_lo += __shfl_xor_sync(0xffffffffu, s_lo, off);
          s_hi += __shfl_xor_sync(0xffffffffu, s_hi, off);
        }
        if (q4 == 0) {
          S.red_sum[c][g8] = s_lo;
          S.red_sum[c][g8 + 8] = s_hi;
        }
        if (c == 0 && q4 == 0) {  // (the first unit's vote always writes them)
          S.m_row[g8] = m_lo;
          S.m_row[g8 + 8] = m_hi;
        }
        named_bar(6, NCT);
        auto lsum = [&](int h) {
          return S.red_sum[0][h] + S.red_sum[1][h] + S.red_sum[2][h] + S.red_sum[3][h];
        };
        const bool full_row = kRows || (seg_kb0 == 0 && kb == upt - 1);
        if (kLse && full_row && c == 0 && q4 == 0) {
          p.lse[t * p.lse_rs + g8] = row_lse2(m_lo, lsum(g8), __ldg(p.sink + g8) * kLog2e);
          p.lse[t * p.lse_rs + g8 + 8] =
              row_lse2(m_hi, lsum(g8 + 8), __ldg(p.sink + g8 + 8) * kLog2e);
        }
        {
          // wait for the segment's MMAs, then read O (this thread: one column
          // per block, all 16 heads)
          wait_or_err(S, S.pv_done[i & 1], (i >> 1) & 1, 12);
          tc_fence_after();
          float f[16];
          if (full_row) {
#pragma unroll
            for (int h = 0; h < 16; ++h)
              f[h] = sink_factor(S.m_row[h], lsum(h), __ldg(p.sink + h) * kLog2e);
          }
          const int64_t pslot = 2 * g + (t == t_first ? 0 : 1);
          __nv_bfloat16* ob = p.o + tb * p.o_sb + tm * p.o_sm;
          float* pacc = p.part_acc + pslot * kPartAccFloats;
#pragma unroll 1
          for (int jb = 0; jb < 4; ++jb) {
            const int col = 128 * jb + 32 * c + lane;
            float v[16];
            tmem_block(tmem, c, jb, v);
            tmem_wait_ld();
            if (full_row) {
#pragma unroll
              for (int h = 0; h < 16; ++h) ob[h * p.o_sh + col] = __float2bfloat16_rn(v[h] * f[h]);
            } else {
#pragma unroll
              for (int h = 0; h < 16; ++h) pacc[h * kDim + col] = v[h];
            }
          }
          tc_fence_before();
          if (!full_row) {
            if (tt < 16) {
              p.part_ml[pslot * kPartMlFloats + tt] = S.m_row[tt];
              p.part_ml[pslot * kPartMlFloats + kHeads + tt] = lsum(tt);
            }
            const int64_t ts = t * upt;
            const int64_t f0 = cta_of_unit(ts, p.units, G);
            if (p.merge_in_kernel) {
              const int np = static_cast<int>(cta_of_unit(ts + upt - 1, p.units, G) - f0 + 1);
              __threadfence();
              named_bar(5, NCT);
              if (tt == 0 && atomicAdd(p.tickets + f0, 1) == np - 1) {
                p.tickets[f0] = 0;
                S.merge_row[S.n_merge++] = t;  // merged after the last unit
              }
            }
          }
        }
        // the next segment's first MMAs overwrite O: every thread's TMEM
        // reads above come first (the next unit's P barrier orders them)
      }
      if (seg_end) ++seg;
      seg_first = seg_end;
      if (++kb == nu_t) {
        kb = 0;
        if constexpr (kRows) {
          t = snake_row(++sk, g, G, R);
          nu_t = nu_n;
          nu_n = units_of_row(p, snake_row(sk + 1, g, G, R));
        } else {
          ++t;
        }
      }
    }
    // Before the tensor memory is freed: the last MMAs are done (bounded;
    // they were issued whatever happened) and, after an error, the last Q
    // load issued has landed.
    if (tt == 0 && n > 0) {
      const uint32_t pb = smem_u32(&S.pv_done[(n - 1) & 1]);
      for (uint32_t k = 0; k < kSpinLimit && !mbar_try_wait(pb, ((n - 1) >> 1) & 1); ++k) {
      }
    }
    if (tt == 0 && q_issued > 0 && *reinterpret_cast<volatile int*>(&S.err) != 0) {
      const uint32_t qb = smem_u32(&S.q_full);
      for (uint32_t k = 0; k < kSpinLimit && !mbar_try_wait(qb, (q_issued - 1) & 1); ++k) {
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc<kTmemCols>(tmem);
  // ---- split rows this CTA merges (ticket mode), from the stored partials
  if (S.n_merge > 0) {
    __threadfence();
    for (int r = 0; r < S.n_merge; ++r) {
      const int64_t tr = S.merge_row[r], ts = tr * p.upt;
      const int64_t f = cta_of_unit(ts, p.units, G);
      const int np = static_cast<int>(cta_of_unit(ts + p.upt - 1, p.units, G) - f + 1);
      const bool f_mid = unit_begin(f, p.units, G) < ts;
#pragma unroll
      for (int k0 = 0; k0 < kHeads * (kDim / 8); k0 += 4 * NT) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = k0 + e * NT + tid;
          merge_split_row(p, f, np, f_mid, tr, k / (kDim / 8), (k % (kDim / 8)) * 8);
        }
      }
    }
  }
}

}  // namespace wt_path

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int wt_unit_keys() { return wt_path::UK; }

int read_wt_index_faults(unsigned long long* out, bool reset) {
  return index_fault_io(sa_wt_index_faults, out, reset);
}

int read_wt_error(int* flags) {
  int v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, sa_wt_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  *flags = v;
  return 0;
}

int reset_wt_error() {
  const int zero = 0;
  return (int)cudaMemcpyToSymbol(sa_wt_error, &zero, sizeof(int));
}

cudaError_t encode_q_map(const Params& p, CUtensorMap* q_map);  // sa_tc.cu

cudaError_t launch_wt(const Params& p, cudaStream_t st) {
  using namespace wt_path;
  CUtensorMap q_map;
  cudaError_t e = encode_q_map(p, &q_map);
  if (e != cudaSuccess) return e;
  static PerDeviceOnce attr_once;
  e = once_per_device(attr_once, [] {
    for (auto* k : {sa_wt_fwd_kernel<false, false>, sa_wt_fwd_kernel<true, false>,
                    sa_wt_fwd_kernel<false, true>, sa_wt_fwd_kernel<true, true>}) {
      const cudaError_t e1 =
          cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
      if (e1 != cudaSuccess) return e1;
    }
    return cudaSuccess;
  });
  if (e != cudaSuccess) return e;
  const bool rows = p.row_units != nullptr;
  if (rows) {
    e = launch_row_units(p, st);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto* kern = p.lse != nullptr ? (rows ? sa_wt_fwd_kernel<true, true> : sa_wt_fwd_kernel<true, false>)
                                : (rows ? sa_wt_fwd_kernel<false, true> : sa_wt_fwd_kernel<false, false>);
  e = cudaLaunchKernelEx(&cfg, kern, p, q_map);
  if (e != cudaSuccess || p.merge_in_kernel || rows) return e;
  return launch_combine(p, st);
}

}  // namespace sa
