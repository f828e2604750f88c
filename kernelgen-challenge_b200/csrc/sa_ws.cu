// sa_ws.cu — warp-specialized persistent gather-attend kernel for sm_100a:
// TMA + cp.async + mbarrier pipeline feeding four consumer warps that run
// both products on the warp-level tensor-core instructions (mma.sync
// m16n8k16).  This is the default variant.
//
// Algorithm: track-01/submission.py:276-347 (math of reference.py:24-40);
// masking of submission.py:313-322; sink in the denominator only
// (submission.py:340-345).  Work schedule and split/combine: sa_common.cuh.
//
// Why warp MMAs here: with 16 heads, one m16n8k16 exactly covers the heads,
// while a tcgen05.mma needs M >= 64, so the heads must sit on N=16, where it
// costs ~60 cycles per instruction (measured for any M in {64,128}, N <= 128).
// Per 64-key unit that is ~2400 tensor cycles (S^T on tcgen05 + P.V) against
// ~1000 for 512 m16n8k16 (S and P.V), and the single tcgen05 issuing thread
// kept each ring slot busy ~3.9 us instead of ~1 us.  The gather, not the
// math, bounds this op; a short slot hold keeps two or more units in flight.
//
// Per 64-key unit (64 KiB of gathered rows, 8 slabs of [64 keys x 64 cols]
// in the 128-byte swizzle):
//   S[16 x 64] = Q[16 x 512] . K^T   consumer warp c: keys 16c..16c+15
//                                    (64 MMAs, Q fragments held in registers
//                                    for the whole row)
//   online softmax on the MMA fragments (running max raised only when a
//   score exceeds it by more than 2^8: one barrier vote per unit)
//   P -> shared memory (bf16, swizzled rows)
//   O[16 x 128c..128c+127] += P . V  consumer warp c: slabs 2c, 2c+1 (64 MMAs)
//   row sums l = P . 1               (4 MMAs, every warp, no reduction)
//
// Warp roles (256 threads, one CTA per SM):
//   warps 0..3   KV producer (cp.async from 128 threads into a 3-deep ring of
//                64 KiB slots)
//   warps 4..7   consumers c = 0..3; once all four hold a row's Q fragments,
//                one of them refills the Q tile with the next row's Q by TMA
//                (one box per 64 columns), so that load overlaps this row
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error code
// in sa_ws_error (readable through sa_device_status) and stops issuing work.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "sa_tc.cuh"

namespace sa {

__device__ int sa_ws_error;  // nonzero after a bounded wait gave up
__device__ unsigned long long sa_ws_index_faults;  // out-of-range indices seen


namespace ws_path {
using namespace tc;

constexpr int UK = 64;                      // keys per unit
constexpr int NSLOT = 3;                    // ring depth (units)
constexpr int SLOT_BYTES = UK * kDim * 2;   // 64 KiB
constexpr int SLAB_BYTES = UK * 128;        // [64 keys x 64 cols] = 8 KiB
constexpr int Q_BYTES = kHeads * kDim * 2;  // 16 KiB
constexpr int P_BYTES = kHeads * UK * 2;    // 2 KiB, P [head][key] bf16
constexpr int NCW = 4;                      // consumer warps
constexpr int NCT = NCW * 32;
constexpr int NT = 4 * 32 + NCT;            // 256: every warp may use 255 registers
constexpr float kRescaleThreshold = 8.0f;   // log2 domain

struct __align__(1024) Smem {
  uint8_t ring[NSLOT][SLOT_BYTES];
  uint8_t q[Q_BYTES];
  uint8_t p[P_BYTES];
  uint32_t mask[NSLOT][2];  // validity: [0] keys 2l, [1] keys 2l+1 (bit l)
  float red_max[NCW][kHeads];
  // full: rows landed (128 cp.async arrivals + mask writer); empty: the four
  // consumer warps finished the unit; q_full: the Q tile of the next row
  uint64_t full[NSLOT], empty[NSLOT], q_full;
  int err;
  uint32_t spin;  // polls before a wait gives up
  // split rows this CTA merges after its last unit (at most its first and last row)
  int n_merge;
  int64_t merge_row[2];
  int n_units;  // row schedule: units of this CTA
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + manual 1 KiB alignment

__device__ __forceinline__ void set_err(Smem& S, int code) {
  if (atomicCAS(&S.err, 0, code) == 0) atomicCAS(&sa_ws_error, 0, code);
}

// Bounded wait that also gives up at once when another warp recorded an error.
// After an error every role keeps walking its loop (so all threads reach the
// same named barriers) but issues no more copies.
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

// Byte offset of the 16-byte chunk `ch` (keys 8ch..8ch+7) of P row `h`:
// rows of 128 B with chunks XOR-swizzled by the row, so ldmatrix reads of 8
// rows hit 8 different bank groups.
__device__ __forceinline__ uint32_t p_chunk(int h, int ch) {
  return h * 128 + ((ch ^ (h & 7)) << 4);
}

// Units per row for the row schedule: ceil((last valid slot + 1) / UK), at
// least 1 (a row without a valid slot still writes o = 0).  Slots past that
// point are masked padding: the forward kernel skips them, and the
// out-of-range indices among them are counted here instead.  One warp per
// row.
__global__ void __launch_bounds__(256) sa_row_units_kernel(const Params p, int* row_units) {
  const int64_t R = p.b * p.m;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const int64_t tb = r / p.m, tm = r - tb * p.m;
  const int32_t* row = p.idx + tb * p.i_sb + tm * p.i_sm;
  int64_t last = -1;
  const bool vec = p.i_sk == 1 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  if (vec) {
    const int64_t nv = p.topk / 4;
#pragma unroll 4
    for (int64_t v = lane; v < nv; v += 32) {
      const int4 w = __ldg(reinterpret_cast<const int4*>(row) + v);
      if (w.x >= 0 && (int64_t)w.x < p.kv_len) last = 4 * v;
      if (w.y >= 0 && (int64_t)w.y < p.kv_len) last = 4 * v + 1;
      if (w.z >= 0 && (int64_t)w.z < p.kv_len) last = 4 * v + 2;
      if (w.w >= 0 && (int64_t)w.w < p.kv_len) last = 4 * v + 3;
    }
    for (int64_t k = 4 * nv + lane; k < p.topk; k += 32) {
      const int32_t id = __ldg(row + k);
      if (id >= 0 && (int64_t)id < p.kv_len) last = k;
    }
  } else {
    for (int64_t k = lane; k < p.topk; k += 32) {
      const int32_t id = __ldg(row + k * p.i_sk);
      if (id >= 0 && (int64_t)id < p.kv_len) last = k;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const int64_t o = __shfl_xor_sync(0xffffffffu, last, off);
    last = o > last ? o : last;
  }
  const int64_t nu = last < 0 ? 1 : (last + UK) / UK;
  if (lane == 0) row_units[r] = static_cast<int>(nu);
  uint32_t faults = 0;
  for (int64_t k = nu * UK + lane; k < p.topk; k += 32)
    faults += index_fault(__ldg(row + k * p.i_sk), p.kv_len) ? 1u : 0u;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) faults += __shfl_xor_sync(0xffffffffu, faults, off);
  if (lane == 0 && faults != 0) atomicAdd(&sa_ws_index_faults, (unsigned long long)faults);
}

// kLse: also write the row log-sum-exp (training forward); a separate
// instance, so the inference kernel carries no trace of it.  kRows: the row
// schedule above instead of contiguous unit ranges (no split rows).
// kGatherOnly (diagnostic, SA_OPT_GATHER_ONLY): the same pipeline, but the
// consumers release each unit as soon as it lands and compute nothing; the
// output is left unwritten.  Its time is the gather's share of the kernel.
// kGroups: several head groups in one launch (Params::hg, blockIdx.y = the
// group); separate instances, since the group offsets alone cost the
// single-group kernel 6-10 % at decode and MTP shapes.
template <bool kLse, bool kRows, bool kGatherOnly = false, bool kGroups = false>
__global__ void __launch_bounds__(NT, 1)
    sa_ws_fwd_kernel(const Params p, const __grid_constant__ CUtensorMap q_map) {
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
  // the combine kernel of split rows may launch now; it waits for this grid
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (tid == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(smem_u32(&S.full[s]), 128 + 1);
      mbar_init(smem_u32(&S.empty[s]), NCW);
    }
    mbar_init(smem_u32(&S.q_full), 1);
    S.err = 0;
    S.spin = p.spin != 0u ? p.spin : kSpinLimit;
    S.n_merge = 0;
    S.n_units = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) tma_prefetch_desc(&q_map);
  // launched as a programmatic dependent of the previous kernel in the stream:
  // the set-up above overlaps its tail; inputs are read only after it is done
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (kRows) {
    // units of this CTA: the row-unit counts are the previous grid's output;
    // every thread loads those of every NT-th row, all loads in flight at once
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
  __syncthreads();
  if constexpr (kRows) n = S.n_units;

  if (warp < 4) {
    // ------------------------------------------------------------ KV producer
    // 128 threads; thread pt copies 16-byte chunk c = pt & 63 of the 32 rows
    // of parity pt >> 6, so every warp-wide cp.async reads 512 contiguous bytes
    // of one row.  The rows land in the 128-byte-swizzled slab layout.  (With
    // half as many issuing threads the gather rate drops by a quarter: issue,
    // not memory, would then bound it.)
    const uint64_t pol = l2_policy_kv(p.kv_policy);
    const int c = tid & 63, par = tid >> 6, j = c >> 3, cc = c & 7;
    int64_t t = t_first, kb = kb_first;
    int64_t tb = t / p.m, tm = t - tb * p.m;
    // row schedule: this row's units, the next row's (loaded a row ahead)
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
      // advance the cursor and prefetch the next unit's indices
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
          count_index_faults(&sa_ws_index_faults, __popc(fa) + __popc(fb));
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
      // the slot's full barrier counts 128 hardware arrivals (one per thread,
      // when its copies land) plus the mask writer's release arrival
      cp_async_mbar_arrive_noinc(smem_u32(&S.full[slot]));
      // (failure-path test: the first slot's release is withheld, so the
      // consumers' wait on it runs out)
      if (warp == 0 && lane == 0 && !(p.test_stall && i == 0)) mbar_arrive(smem_u32(&S.full[slot]));
    }
    cp_async_wait<0>();
  } else {
    // ------------------------------------------------------------ consumers
    const int c = warp - 4;                   // 0..3
    const int tt = tid - 128;                 // consumer thread 0..127
    const int g8 = lane >> 2, q4 = lane & 3;  // mma fragment coordinates
    const uint32_t qbase = smem_u32(S.q), pbase = smem_u32(S.p);
    const uint32_t kOnes = 0x3F803F80u;  // bf16 pair (1, 1)
    uint32_t qf[32][4];                  // Q A-fragments, 32 k-steps of 16 columns
    float m_lo = -INFINITY, m_hi = -INFINITY;  // running max, heads g8 / g8+8 (log2)
    float o[16][4];  // O[heads g8, g8+8][128c + 8nt + 2q4 + {0,1}]
    float lacc[4];   // running row sums: [0] head g8, [2] head g8+8
    // Q loads issued by consumer thread 0; after an error none is issued, and
    // the one possibly in flight is waited for before the CTA exits.
    int q_issued = 0;
    auto issue_q = [&](int64_t row) {
      if (*reinterpret_cast<volatile int*>(&S.err) != 0) return;
      ++q_issued;
      const int64_t qb = row / p.m, qm = row - qb * p.m;
      fence_proxy_async_smem();  // the Q fragment reads above precede the TMA refill
      mbar_arrive_expect_tx(smem_u32(&S.q_full), Q_BYTES);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        tma_load_4d(qbase + j * 2048, &q_map, 64 * j, kGroups ? kHeads * (int32_t)blockIdx.y : 0, (int32_t)qm, (int32_t)qb,
                    smem_u32(&S.q_full));
    };
    if (tt == 0) issue_q(t_first);
    int64_t t = t_first, kb = kb_first, seg_kb0 = kb_first;
    int64_t sk = 0, nu_t = upt, nu_n = 0;  // as in the producer
    if constexpr (kRows) {
      nu_t = units_of_row(p, t);
      nu_n = units_of_row(p, snake_row(1, g, G, R));
    }
    int seg = 0;
    bool seg_first = true;
    for (int i = 0; i < n; ++i) {
      const bool seg_end = (i == n - 1) || kb == nu_t - 1;
      if (seg_first) {
        m_lo = m_hi = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
        lacc[0] = lacc[1] = lacc[2] = lacc[3] = 0.f;
        seg_kb0 = kb;
        // this row's Q into registers; once every consumer holds it, the tile
        // is refilled with the next row's Q (one TMA box per 64 columns)
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
      if constexpr (kGatherOnly) {
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&S.empty[slot]));
      } else {
      const uint32_t sb = smem_u32(S.ring[slot]);

      // ---- S for keys 16c + 8nt + {0..7}: 2 n-tiles x 32 k-steps, 2-way split
      float sa[2][2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int z = 0; z < 2; ++z) sa[nt][z][0] = sa[nt][z][1] = sa[nt][z][2] = sa[nt][z][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < 16; ++kp) {  // k-steps 2kp, 2kp+1: columns 32kp..32kp+31
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
      // ---- softmax on the fragments: x[nt][0,1] head g8, x[nt][2,3] head g8+8,
      //      keys 16c + 8nt + 2q4 + {0,1}
      const uint32_t mw0 = S.mask[slot][0], mw1 = S.mask[slot][1];
      float x[2][4];
      bool over = false;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int l = 8 * c + 4 * nt + q4;  // producer lane that loaded these keys
        const bool v0 = (mw0 >> l) & 1u, v1 = (mw1 >> l) & 1u;
        x[nt][0] = v0 ? (sa[nt][0][0] + sa[nt][1][0]) * p.scale_log2 : -INFINITY;
        x[nt][1] = v1 ? (sa[nt][0][1] + sa[nt][1][1]) * p.scale_log2 : -INFINITY;
        x[nt][2] = v0 ? (sa[nt][0][2] + sa[nt][1][2]) * p.scale_log2 : -INFINITY;
        x[nt][3] = v1 ? (sa[nt][0][3] + sa[nt][1][3]) * p.scale_log2 : -INFINITY;
        over |= fmaxf(x[nt][0], x[nt][1]) > m_lo + kRescaleThreshold;
        over |= fmaxf(x[nt][2], x[nt][3]) > m_hi + kRescaleThreshold;
      }
      // The vote barrier also orders this unit's P writes after every warp's
      // P.V of the previous unit (single P tile).
      if (named_bar_or(1, NCT, over)) {
        // raise the running max to the block max (rare after a row's first unit)
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
      {
        const float base_lo = (m_lo == -INFINITY) ? 0.f : m_lo;
        const float base_hi = (m_hi == -INFINITY) ? 0.f : m_hi;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int ch = 2 * c + nt;  // keys 8ch..8ch+7
          *reinterpret_cast<uint32_t*>(S.p + p_chunk(g8, ch) + 4 * q4) =
              pack_bf16x2(exp2f(x[nt][0] - base_lo), exp2f(x[nt][1] - base_lo));
          *reinterpret_cast<uint32_t*>(S.p + p_chunk(g8 + 8, ch) + 4 * q4) =
              pack_bf16x2(exp2f(x[nt][2] - base_hi), exp2f(x[nt][3] - base_hi));
        }
      }
      named_bar(3, NCT);  // P of all 64 keys written

      // ---- O[16 x 128 cols of this warp] += P[16 x 64] . V[64 x 128]
#pragma unroll
      for (int kst = 0; kst < 4; ++kst) {
        uint32_t pa[4];
        {
          const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
          ldmatrix_x4(pa, pbase + p_chunk(row, 2 * kst + (lane >> 4)));
        }
        mma_16816(lacc, pa, kOnes, kOnes);  // row sums of the bf16 P actually used
        const int kr = kst * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          const int slab = 2 * c + (np >> 2);
          const int ch = ((np & 3) << 1) + (lane >> 4);
          uint32_t vb[4];
          ldmatrix_x4_trans(vb, sb + slab * SLAB_BYTES + kr * 128 + ((ch ^ (kr & 7)) << 4));
          mma_16816(o[2 * np], pa, vb[0], vb[1]);
          mma_16816(o[2 * np + 1], pa, vb[2], vb[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.empty[slot]));  // slot free for the producer

      if (seg_end) {
        // ---------------- epilogue of the segment ending at unit i ----------
        const int64_t tb = t / p.m, tm = t - tb * p.m;
        const float l_lo = lacc[0], l_hi = lacc[2];
        const int hy = kGroups ? kHeads * (int)blockIdx.y : 0;  // first head of this CTA's group
        if (kRows || (seg_kb0 == 0 && kb == upt - 1)) {
          const float f_lo = sink_factor(m_lo, l_lo, __ldg(p.sink + hy + g8) * kLog2e);
          const float f_hi = sink_factor(m_hi, l_hi, __ldg(p.sink + hy + g8 + 8) * kLog2e);
          if (kLse && c == 0 && q4 == 0) {
            float* lr = p.lse + t * p.lse_rs + hy;
            lr[g8] = row_lse2(m_lo, l_lo, __ldg(p.sink + hy + g8) * kLog2e);
            lr[g8 + 8] = row_lse2(m_hi, l_hi, __ldg(p.sink + hy + g8 + 8) * kLog2e);
          }
          __nv_bfloat16* ob = p.o + tb * p.o_sb + tm * p.o_sm + hy * p.o_sh;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt) {
            const int d = 128 * c + 8 * nt + 2 * q4;
            *reinterpret_cast<uint32_t*>(ob + g8 * p.o_sh + d) =
                pack_bf16x2(o[nt][0] * f_lo, o[nt][1] * f_lo);
            *reinterpret_cast<uint32_t*>(ob + (g8 + 8) * p.o_sh + d) =
                pack_bf16x2(o[nt][2] * f_hi, o[nt][3] * f_hi);
          }
        } else {
          const int64_t pslot = 2 * (kGroups ? g + G * blockIdx.y : g) + (t == t_first ? 0 : 1);
          float* pacc = p.part_acc + pslot * kPartAccFloats;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt) {
            const int d = 128 * c + 8 * nt + 2 * q4;
            *reinterpret_cast<float2*>(pacc + g8 * kDim + d) = make_float2(o[nt][0], o[nt][1]);
            *reinterpret_cast<float2*>(pacc + (g8 + 8) * kDim + d) =
                make_float2(o[nt][2], o[nt][3]);
          }
          if (c == 0 && q4 == 0) {
            p.part_ml[pslot * kPartMlFloats + g8] = m_lo;
            p.part_ml[pslot * kPartMlFloats + g8 + 8] = m_hi;
            p.part_ml[pslot * kPartMlFloats + kHeads + g8] = l_lo;
            p.part_ml[pslot * kPartMlFloats + kHeads + g8 + 8] = l_hi;
          }
          // In-kernel merge: the row's CTAs f..last each take a ticket once
          // their part is stored; the last to arrive merges the row (nothing
          // waits) and zeroes the ticket word for the next call.  Otherwise
          // the combine kernel merges the split rows after this grid.
          if (p.merge_in_kernel) {
            const int64_t ts = t * upt;
            const int64_t f = cta_of_unit(ts, p.units, G);
            const int np = static_cast<int>(cta_of_unit(ts + upt - 1, p.units, G) - f + 1);
            __threadfence();
            named_bar(5, NCT);
            int* tk = p.tickets + (kGroups ? G * blockIdx.y : 0) + f;
            if (tt == 0 && atomicAdd(tk, 1) == np - 1) {
              *tk = 0;
              S.merge_row[S.n_merge++] = t;  // merged after the last unit (registers free)
            }
          }
        }
      }
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
    // After an error the last Q load issued may still be in flight: wait for
    // it (its phase is the only one not yet seen) before the CTA exits.
    if (tt == 0 && q_issued > 0 && *reinterpret_cast<volatile int*>(&S.err) != 0) {
      const uint32_t qb = smem_u32(&S.q_full);
      for (uint32_t k = 0; k < kSpinLimit && !mbar_try_wait(qb, (q_issued - 1) & 1); ++k) {
      }
    }
  }
  // ---- every thread (the producers are idle by now) merges the split rows
  // whose last part this CTA stored: 1024 (head, 8-column) items per row,
  // four per thread, their loads in flight together
  __syncthreads();
  if (S.n_merge > 0) {
    __threadfence();
    const Params gp = kGroups ? group_params(p, blockIdx.y) : p;
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
          merge_split_row(gp, f, np, f_mid, tr, k / (kDim / 8), (k % (kDim / 8)) * 8);
        }
      }
    }
  }
}

}  // namespace ws_path

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int ws_unit_keys() { return ws_path::UK; }


int read_ws_index_faults(unsigned long long* out, bool reset) {
  return index_fault_io(sa_ws_index_faults, out, reset);
}

int read_ws_error(int* flags) {
  int v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, sa_ws_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  *flags = v;
  return 0;
}

int reset_ws_error() {
  const int zero = 0;
  return (int)cudaMemcpyToSymbol(sa_ws_error, &zero, sizeof(int));
}

cudaError_t encode_q_map(const Params& p, CUtensorMap* q_map);  // sa_tc.cu

// A plain launch: it follows the previous op in the stream, and the forward
// kernel after it waits for it (griddepcontrol.wait) before reading counts.
cudaError_t launch_row_units(const Params& p, cudaStream_t st) {
  const int64_t R = p.b * p.m;
  ws_path::sa_row_units_kernel<<<static_cast<unsigned>((R + 7) / 8), 256, 0, st>>>(
      p, const_cast<int*>(p.row_units));
  return cudaGetLastError();
}

cudaError_t launch_ws(const Params& p, cudaStream_t st) {
  using namespace ws_path;
  CUtensorMap q_map;
  cudaError_t e = encode_q_map(p, &q_map);
  if (e != cudaSuccess) return e;
  static PerDeviceOnce attr_once;
  e = once_per_device(attr_once, [] {
    for (auto* k : {sa_ws_fwd_kernel<false, false>, sa_ws_fwd_kernel<true, false>,
                    sa_ws_fwd_kernel<false, true>, sa_ws_fwd_kernel<true, true>,
                    sa_ws_fwd_kernel<false, false, true>, sa_ws_fwd_kernel<false, true, true>,
                    sa_ws_fwd_kernel<false, false, false, true>,
                    sa_ws_fwd_kernel<true, false, false, true>,
                    sa_ws_fwd_kernel<false, true, false, true>,
                    sa_ws_fwd_kernel<true, true, false, true>}) {
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
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid), static_cast<unsigned>(p.hg), 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto* kern = p.lse != nullptr ? (rows ? sa_ws_fwd_kernel<true, true> : sa_ws_fwd_kernel<true, false>)
                                : (rows ? sa_ws_fwd_kernel<false, true> : sa_ws_fwd_kernel<false, false>);
  if (p.hg > 1)
    kern = p.lse != nullptr
               ? (rows ? sa_ws_fwd_kernel<true, true, false, true>
                       : sa_ws_fwd_kernel<true, false, false, true>)
               : (rows ? sa_ws_fwd_kernel<false, true, false, true>
                       : sa_ws_fwd_kernel<false, false, false, true>);
  else if (opt_gather_only() && p.lse == nullptr)
    kern = rows ? sa_ws_fwd_kernel<false, true, true> : sa_ws_fwd_kernel<false, false, true>;
  e = cudaLaunchKernelEx(&cfg, kern, p, q_map);
  if (e != cudaSuccess || p.merge_in_kernel || rows) return e;
  return launch_combine(p, st);
}

}  // namespace sa
