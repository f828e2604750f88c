// sa_fp8.cu — sparse_attn over an fp8 (e4m3) KV cache with one fp32 scale per
// token, for sm_100a.  Same warp-specialized pipeline as sa_ws.cu, but every
// gathered row is 512 B instead of 1 KiB.
//
// Semantics: the bf16 op applied to the dequantised cache
//   kv[b, t, :] = kv8[b, t, :] * kscale[b, t]
// (track-01/reference/reference.py:24-40 on that kv; masking of
// track-01/submission.py:313-322; sink in the denominator only).  The
// reference has no fp8 cache.  This is the fp8 KV-cache layout variant.
//
// Arithmetic: both products are f16 warp MMAs (mma.sync m16n8k16, fp32
// accumulate).  The e4m3 K and V values are widened to f16 in registers
// (cvt.f16x2.e4m3x2, exact) right before each MMA, so shared memory and HBM
// only ever hold the 1-byte values.  The e4m3 MMA (m16n8k32) was measured
// here at the same FLOP rate as m16n8k16 (about twice the cycles for twice
// the work), and it would need Q and P in e4m3.  The f16 path keeps them at
// full precision for the same tensor time.
//   Q:   bf16 -> f16 after scaling each head by a power of two that puts its
//        amax in [2^14, 2^15): exact, since f16 has more mantissa bits than
//        bf16 (values below amax * 2^-28 would lose bits).
//   S:   (Q.K8) * 2^-e_h * kscale[key] * scale, fp32.
//   P:   f16 (11 significant bits).  For V the weights are
//        Pv = P * kscale[key] / R, where R is a running maximum of the row's
//        token scales, so Pv <= P <= 2^8.  O is kept in units of R and
//        rescaled when R grows.
//   l:   P . 1 on the same f16 P, without the token scales.
//
// Per 64-key unit (32 KiB of gathered rows + 64 scales), consumer warp c:
//   S for keys 16c..16c+15: 2 n-tiles x 32 k16-steps = 64 MMAs.  An ldmatrix
//     of the e4m3 rows gives each lane columns 4q..4q+3 of one key per 16-column
//     step.  Widened, they are the lane's two B registers if the k index is
//     permuted within the step (k 2q,2q+1 <-> columns 4q,4q+1 and k 2q+8,2q+9
//     <-> 4q+2,4q+3).  Q is stored in shared memory with the same column
//     permutation, so its ldmatrix A-fragments match.
//   O for columns 128c..128c+127: 4 k16-steps x 16 n-tiles = 64 MMAs.  The B
//     fragment of V needs two keys of one column per register; the rows hold
//     one key's columns.  A lane reads 32-bit words (4 columns) of its keys
//     2q, 2q+1, 2q+8, 2q+9, pairs the keys bytewise (prmt) and widens each
//     pair.  So output n-tile j of column group G holds columns 32G + 4n + j,
//     not 32G + 8j + n: a fixed column permutation, undone at the store.
//
// Warp roles (256 threads, one CTA per SM), as in sa_ws.cu:
//   warps 0..3   producer: cp.async of 64 rows x 512 B per unit (each warp-wide
//                instruction reads one row) into a 5-deep ring; warp 0 also
//                writes the unit's validity mask, token scales and their max
//   warps 4..7   consumers; consumer thread 0 refills the bf16 Q tile by TMA
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error code
// in sa_fp8_error (readable through sa_device_status) and stops issuing work.
#include <type_traits>
#include <cuda.h>
#include <cuda_fp16.h>

#include "sa_tc.cuh"

namespace sa {

__device__ int sa_fp8_error;                        // nonzero after a bounded wait gave up
__device__ unsigned long long sa_fp8_index_faults;  // out-of-range indices seen

namespace fp8_path {
using namespace tc;

constexpr int UK = 64;                      // keys per unit
constexpr int NSLOT = 5;                    // ring depth (units)
constexpr int ROW_BYTES = kDim;             // one e4m3 row
constexpr int SLOT_BYTES = UK * ROW_BYTES;  // 32 KiB
constexpr int Q_BYTES = kHeads * kDim * 2;  // 16 KiB (bf16 TMA tile, f16 MMA tile)
constexpr int QH_ROW = kDim * 2;            // f16 Q row: 1 KiB
constexpr int PT_BYTES = kHeads * UK * 2;   // 2 KiB f16 P tile [head][key]
constexpr int NCW = 4;                      // consumer warps
constexpr int NCT = NCW * 32;
constexpr int NT = 4 * 32 + NCT;            // 256
constexpr float kRescaleThreshold = 8.0f;   // log2 domain: P <= 2^8
constexpr float kE4m3Max = 448.0f;
constexpr uint32_t kOnesF16 = 0x3C003C00u;  // f16 pair (1, 1)

struct __align__(1024) Smem {
  uint8_t ring[NSLOT][SLOT_BYTES];  // rows of 512 B, 16-byte chunks swizzled by row
  uint8_t q[Q_BYTES];               // bf16 Q: 8 TMA boxes [16 heads][64 cols], 128-byte swizzle
  uint8_t qh[Q_BYTES];              // f16 Q [16][512], columns permuted per 16, rows swizzled
  uint8_t pl[PT_BYTES];             // f16 P for the row sums
  uint8_t pv[PT_BYTES];             // f16 P * kscale / R for P.V
  float kscale[NSLOT][UK];          // token scales of the unit (0 for masked slots)
  float kmax[NSLOT];                // their maximum
  uint32_t mask[NSLOT][2];          // validity: [0] keys 2l, [1] keys 2l+1 (bit l)
  float red_max[NCW][kHeads];
  // full: rows landed (128 cp.async arrivals + warp 0's release arrival);
  // empty: the four consumer warps finished the unit; q_full: next row's Q
  uint64_t full[NSLOT], empty[NSLOT], q_full;
  int err;
  uint32_t spin;  // polls before a wait gives up
  // split rows this CTA merges after its last unit (at most its first and last row)
  int n_merge;
  int64_t merge_row[2];
  int n_units;  // row schedule: units of this CTA
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + manual 1 KiB alignment
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ void set_err(Smem& S, int code) {
  if (atomicCAS(&S.err, 0, code) == 0) atomicCAS(&sa_fp8_error, 0, code);
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

// Byte offset of 16-byte chunk `ch` (0..31) of gathered row `r` in a slot:
// chunks XOR-swizzled by r & 7, so ldmatrix of 8 consecutive rows at one chunk
// and the V reads of rows 2i + d (i = 0..3) at one chunk pair are both
// conflict-free.
__device__ __forceinline__ uint32_t row_chunk(int r, int ch) {
  return r * ROW_BYTES + ((ch ^ (r & 7)) << 4);
}

// f16 Q tile: row h (1 KiB), 16-byte chunk ch (0..63) swizzled by h & 7.
// Chunk 2j holds columns 16j + 4i + {0,1} and chunk 2j+1 columns
// 16j + 4i + {2,3} (i = 0..3, two f16 each).
__device__ __forceinline__ uint32_t qh_chunk(int h, int ch) {
  return h * QH_ROW + ((ch ^ (h & 7)) << 4);
}

// f16 P tile: row h (128 B), chunk ch = keys 8ch..8ch+7, swizzled by h & 7.
__device__ __forceinline__ uint32_t p_chunk(int h, int ch) {
  return h * 128 + ((ch ^ (h & 7)) << 4);
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Four e4m3 (bytes of w, low first) -> two f16 pairs: lo = (b0, b1), hi = (b2, b3).
__device__ __forceinline__ void widen4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n cvt.rn.f16x2.e4m3x2 %0, l;\n"
      " cvt.rn.f16x2.e4m3x2 %1, h;\n}\n"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

// Two fp32 -> e4m3 (round to nearest even, saturating), x0 in the low byte.
__device__ __forceinline__ uint16_t e4m3x2(float x0, float x1) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(r) : "f"(x1), "f"(x0));
  return r;
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];\n" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(addr), "r"(v));
}

// Four bf16 of the TMA Q tile: head h, columns col..col+3 (col % 4 == 0).
__device__ __forceinline__ float4 q_four(uint32_t qbase, int h, int col) {
  const int box = col >> 6, cb = col & 63;
  const uint32_t addr = qbase + box * 2048 + h * 128 + (((cb >> 3) ^ (h & 7)) << 4) + (cb & 7) * 2;
  uint32_t w0, w1;
  asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];\n" : "=r"(w0), "=r"(w1) : "r"(addr));
  const float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w0));
  const float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w1));
  return make_float4(a.x, a.y, b.x, b.y);
}

// 2^e as a float for e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

struct Cursor {
  int64_t kb, tb, tm;
  __device__ __forceinline__ void advance(int64_t upt, int64_t m) {
    if (++kb == upt) {
      kb = 0;
      if (++tm == m) {
        tm = 0;
        ++tb;
      }
    }
  }
};

// kRows: the row schedule of sa_common.cuh (whole rows in snake order, each
// up to its last valid slot) instead of contiguous unit ranges.
template <bool kRows>
__global__ void __launch_bounds__(NT, 1)
    sa_fp8_fwd_kernel(const Params p, const __grid_constant__ CUtensorMap q_map) {
  extern __shared__ uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t G = p.grid, g = blockIdx.x;
  const int64_t nrows = p.b * p.m;
  int64_t u0 = 0, u1 = 0;
  if constexpr (kRows) {
    if (g >= nrows) return;  // (the host keeps rows >= 2G)
  } else {
    u0 = unit_begin(g, p.units, G);
    u1 = unit_begin(g + 1, p.units, G);
    if (u1 <= u0) return;
  }
  int n = static_cast<int>(u1 - u0);  // units of this CTA (row schedule: below)
  const int64_t upt = p.upt;
  const int64_t t_first = kRows ? snake_row(0, g, G, nrows) : u0 / upt;
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
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (kRows) {  // units of this CTA, all row counts loaded at once
    __syncthreads();      // (S.n_units initialised)
    int part = 0;
    for (int64_t k = tid;; k += NT) {
      const int64_t r = snake_row(k, g, G, nrows);
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
    // ------------------------------------------------------------ producer
    // Warp w copies rows w, w+4, ..., w+60 of each unit; lane = 16-byte chunk,
    // so one warp-wide cp.async reads one 512-byte row.  Indices run two
    // units ahead and warp 0's token scales one unit ahead, so neither
    // dependent global load stalls the copy issue.
    const uint64_t pol = l2_policy_kv(p.kv_policy);
    const uint8_t* kv8 = reinterpret_cast<const uint8_t*>(p.kv);
    auto load_ids = [&](const auto& cu, int32_t& a, int32_t& b) {
      const int64_t k0 = cu.kb * UK + 2 * lane;
      const int32_t* base = p.idx + cu.tb * p.i_sb + cu.tm * p.i_sm;
      a = k0 < p.topk ? __ldg(base + k0 * p.i_sk) : -1;
      b = k0 + 1 < p.topk ? __ldg(base + (k0 + 1) * p.i_sk) : -1;
    };
    auto valid = [&](int32_t id) { return id >= 0 && (int64_t)id < p.kv_len; };
    auto load_scales = [&](int64_t tb, int32_t a, int32_t b, float& sa_, float& sb_) {
      const float* base = p.kscale + tb * p.ks_sb;
      sa_ = valid(a) ? __ldg(base + (int64_t)a * p.ks_sn) : 0.f;
      sb_ = valid(b) ? __ldg(base + (int64_t)b * p.ks_sn) : 0.f;
    };
    std::conditional_t<kRows, RowCursor, Cursor> cu;
    if constexpr (kRows) {
      cu.start(p, g, G, nrows);
    } else {
      cu = Cursor{kb_first, t_first / p.m, t_first - (t_first / p.m) * p.m};
    }
    auto advance = [&] {
      if constexpr (kRows) {
        cu.advance(p, g, G, nrows);
      } else {
        cu.advance(upt, p.m);
      }
    };
    int32_t xa0, xb0, xa1 = -1, xb1 = -1;  // indices of units i and i+1
    int64_t tb0 = cu.tb, tb1 = cu.tb;
    float sa0 = 0.f, sb0 = 0.f;           // scales of unit i (warp 0)
    load_ids(cu, xa0, xb0);
    if (warp == 0) load_scales(tb0, xa0, xb0, sa0, sb0);
    advance();
    if (n > 1) {
      load_ids(cu, xa1, xb1);
      tb1 = cu.tb;
    }
    for (int i = 0; i < n; ++i) {
      const int32_t ia = xa0, ib = xb0;
      const float fsa = sa0, fsb = sb0;
      const int64_t cur_tb = tb0;
      xa0 = xa1;
      xb0 = xb1;
      tb0 = tb1;
      advance();  // unit i + 2
      if (i + 2 < n) {
        load_ids(cu, xa1, xb1);
        tb1 = cu.tb;
      }
      if (warp == 0 && i + 1 < n) load_scales(tb0, xa0, xb0, sa0, sb0);

      const int slot = i % NSLOT;
      const bool ok = i < NSLOT || wait_or_err(S, S.empty[slot], ((i / NSLOT) - 1) & 1, 1);
      if (!__all_sync(0xffffffffu, ok)) continue;
      const uint8_t* kvb = kv8 + cur_tb * p.kv_sb + lane * 16;
      const uint32_t dst0 = smem_u32(S.ring[slot]);
      const int32_t mine = (warp & 1) ? ib : ia;  // rows of this warp have parity warp & 1
#pragma unroll 8
      for (int k = 0; k < UK / 4; ++k) {
        const int r = warp + 4 * k;
        const int32_t id = __shfl_sync(0xffffffffu, mine, r >> 1);
        const bool v = valid(id);
        cp_async16_hint(dst0 + row_chunk(r, lane), kvb + (v ? (int64_t)id : 0) * p.kv_sn,
                        v ? 16 : 0, pol);
      }
      cp_async_mbar_arrive_noinc(smem_u32(&S.full[slot]));
      if (warp == 0) {
        const uint32_t ma = __ballot_sync(0xffffffffu, valid(ia));
        const uint32_t mb = __ballot_sync(0xffffffffu, valid(ib));
        const uint32_t fa = __ballot_sync(0xffffffffu, index_fault(ia, p.kv_len));
        const uint32_t fb = __ballot_sync(0xffffffffu, index_fault(ib, p.kv_len));
        *reinterpret_cast<float2*>(&S.kscale[slot][2 * lane]) = make_float2(fsa, fsb);
        float km = fmaxf(fsa, fsb);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) km = fmaxf(km, __shfl_xor_sync(0xffffffffu, km, off));
        if (lane == 0) {
          S.mask[slot][0] = ma;
          S.mask[slot][1] = mb;
          S.kmax[slot] = km;
          count_index_faults(&sa_fp8_index_faults, __popc(fa) + __popc(fb));
        }
        __syncwarp();
        // release: the slot's full barrier also counts this arrival, made
        // after every lane's scale and mask writes
        // (failure-path test: the first slot's release is withheld, so the
        // consumers' wait on it runs out)
        if (lane == 0 && !(p.test_stall && i == 0)) mbar_arrive(smem_u32(&S.full[slot]));
      }
    }
    cp_async_wait<0>();
  } else {
    // ------------------------------------------------------------ consumers
    const int c = warp - 4;                   // 0..3
    const int tt = tid - 128;                 // consumer thread 0..127
    const int g8 = lane >> 2, q4 = lane & 3;  // mma fragment coordinates
    const int mtx = lane >> 3;                // ldmatrix: matrix whose row address this lane gives
    const uint32_t qbase = smem_u32(S.q), qhbase = smem_u32(S.qh);
    const uint32_t plbase = smem_u32(S.pl), pvbase = smem_u32(S.pv);
    float qs_lo = 0.f, qs_hi = 0.f;  // 2^-e * scale * log2(e), heads g8 / g8+8
    float m_lo = -INFINITY, m_hi = -INFINITY;  // running max (log2 domain)
    float R = 0.f, invR = 0.f;       // running max of the token scales seen
    float o[16][4];  // O / R; n-tile 4G+j: heads g8, g8+8, columns 128c+32G+8q4+{j, 4+j}
    float lacc[4];   // running row sums: [0] head g8, [2] head g8+8
    // Q loads issued by consumer thread 0; after an error none is issued, and
    // the one possibly in flight is waited for before the CTA exits.
    int q_issued = 0;
    auto issue_q = [&](int64_t row) {
      if (*reinterpret_cast<volatile int*>(&S.err) != 0) return;
      ++q_issued;
      const int64_t qb = row / p.m, qm = row - qb * p.m;
      fence_proxy_async_smem();  // the Q reads above precede the TMA refill
      mbar_arrive_expect_tx(smem_u32(&S.q_full), Q_BYTES);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        tma_load_4d(qbase + j * 2048, &q_map, 64 * j, 0, (int32_t)qm, (int32_t)qb,
                    smem_u32(&S.q_full));
    };
    if (tt == 0) issue_q(t_first);
    int64_t t = t_first, kb = kb_first, seg_kb0 = kb_first;
    int64_t sk = 0, nu_t = upt, nu_n = 0;  // row schedule: as RowCursor
    if constexpr (kRows) {
      nu_t = units_of_row(p, t);
      nu_n = units_of_row(p, snake_row(1, g, G, nrows));
    }
    int seg = 0;
    bool seg_first = true;
    for (int i = 0; i < n; ++i) {
      const bool seg_end = (i == n - 1) || kb == nu_t - 1;
      if (seg_first) {
        m_lo = m_hi = -INFINITY;
        R = invR = 0.f;
        seg_kb0 = kb;
        wait_or_err(S, S.q_full, seg & 1, 7);
        // This row's Q as f16: warp c converts columns 128c..128c+127 (lane:
        // columns 16j + 4q4..+3 of heads g8, g8+8), after a per-head amax over
        // all four warps' columns.  Once per row: loops kept rolled.
        float a_lo = 0.f, a_hi = 0.f;
#pragma unroll 1
        for (int j = 8 * c; j < 8 * c + 8; ++j) {
          const float4 u = q_four(qbase, g8, 16 * j + 4 * q4);
          const float4 v = q_four(qbase, g8 + 8, 16 * j + 4 * q4);
          a_lo = fmaxf(a_lo, fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))));
          a_hi = fmaxf(a_hi, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
          a_lo = fmaxf(a_lo, __shfl_xor_sync(0xffffffffu, a_lo, off));
          a_hi = fmaxf(a_hi, __shfl_xor_sync(0xffffffffu, a_hi, off));
        }
        if (q4 == 0) {
          S.red_max[c][g8] = a_lo;
          S.red_max[c][g8 + 8] = a_hi;
        }
        named_bar(5, NCT);
#pragma unroll
        for (int w = 0; w < NCW; ++w) {
          a_lo = fmaxf(a_lo, S.red_max[w][g8]);
          a_hi = fmaxf(a_hi, S.red_max[w][g8 + 8]);
        }
        // e: amax * 2^e in [2^14, 2^15) (amax = f * 2^E, f in [0.5, 1): e = 15 - E)
        auto head_exp = [](float a) {
          const int E = ((__float_as_int(a) >> 23) & 0xff) - 126;
          const int e = a > 0.f ? 15 - E : 0;
          return e < -126 ? -126 : (e > 126 ? 126 : e);
        };
        const int e_lo = head_exp(a_lo), e_hi = head_exp(a_hi);
        const float s_lo = exp2i(e_lo), s_hi = exp2i(e_hi);
        qs_lo = exp2i(-e_lo) * p.scale_log2;
        qs_hi = exp2i(-e_hi) * p.scale_log2;
#pragma unroll 1
        for (int j = 8 * c; j < 8 * c + 8; ++j) {
          const float4 u = q_four(qbase, g8, 16 * j + 4 * q4);
          const float4 v = q_four(qbase, g8 + 8, 16 * j + 4 * q4);
          sts32(qhbase + qh_chunk(g8, 2 * j) + 4 * q4, pack_f16x2(u.x * s_lo, u.y * s_lo));
          sts32(qhbase + qh_chunk(g8, 2 * j + 1) + 4 * q4, pack_f16x2(u.z * s_lo, u.w * s_lo));
          sts32(qhbase + qh_chunk(g8 + 8, 2 * j) + 4 * q4, pack_f16x2(v.x * s_hi, v.y * s_hi));
          sts32(qhbase + qh_chunk(g8 + 8, 2 * j + 1) + 4 * q4, pack_f16x2(v.z * s_hi, v.w * s_hi));
        }
        // the f16 tile is complete and the bf16 tile free for the next row.
        // (The previous row's f16 tile reads all came before the previous
        // unit's vote barrier; its red_max reads before its P barrier.)
        named_bar(4, NCT);
        if constexpr (kRows) {
          const int64_t tn = snake_row(sk + 1, g, G, nrows);
          if (tt == 0 && tn >= 0) issue_q(tn);
        } else if (tt == 0 && t < t_last) {
          issue_q(t + 1);
        }
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
        lacc[0] = lacc[1] = lacc[2] = lacc[3] = 0.f;
      }
      const int slot = i % NSLOT;
      wait_or_err(S, S.full[slot], (i / NSLOT) & 1, 8);
      const uint32_t sb = smem_u32(S.ring[slot]);

      // ---- S for keys 16c + 8nt + {0..7}: [nt][0] even k-steps, [nt][1] odd
      float sa[2][2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int z = 0; z < 2; ++z) sa[nt][z][0] = sa[nt][z][1] = sa[nt][z][2] = sa[nt][z][3] = 0.f;
      {
        // K: rows 16c + 8nt + (lane & 7), chunk 4J + mtx gives k16-step 4J + mtx.
        // (4J + mtx) ^ (lane & 7) = 8 (J >> 1) + ((4 (J & 1) + mtx) ^ (lane & 7)).
        uint32_t koff[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int jo = 0; jo < 2; ++jo)
            koff[nt][jo] = sb + (16 * c + 8 * nt + (lane & 7)) * ROW_BYTES +
                           (((4 * jo + mtx) ^ (lane & 7)) << 4);
        // Q: row (lane & 7) + 8 (mtx & 1), chunk 2ks + (mtx >> 1); for ks = 4J + kk
        // the chunk is 8J + (2kk + (mtx >> 1)) and only the low part is swizzled.
        uint32_t qoff[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          qoff[kk] = qhbase + ((lane & 7) + 8 * (mtx & 1)) * QH_ROW +
                     (((2 * kk + (mtx >> 1)) ^ (lane & 7)) << 4);
#pragma unroll
        for (int J2 = 0; J2 < 4; ++J2)
#pragma unroll
          for (int jo = 0; jo < 2; ++jo) {  // J = 2 J2 + jo: k16-steps 4J..4J+3
            uint32_t kf[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) ldmatrix_x4(kf[nt], koff[nt][jo] + (J2 << 7));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              uint32_t qa[4];
              ldmatrix_x4(qa, qoff[kk] + (J2 << 8) + (jo << 7));
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) {
                uint32_t b0, b1;
                widen4(kf[nt][kk], b0, b1);
                mma_f16(sa[nt][kk & 1], qa, b0, b1);
              }
            }
          }
      }
      // ---- softmax on the fragments: x[nt][0,1] head g8, x[nt][2,3] head g8+8,
      //      keys 16c + 8nt + 2q4 + {0,1}
      const uint32_t mw0 = S.mask[slot][0], mw1 = S.mask[slot][1];
      float2 ks[2];
      float x[2][4];
      bool over = false;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int key = 16 * c + 8 * nt + 2 * q4;
        const int l = key >> 1;  // mask bit of this key pair
        ks[nt] = *reinterpret_cast<const float2*>(&S.kscale[slot][key]);
        const bool v0 = (mw0 >> l) & 1u, v1 = (mw1 >> l) & 1u;
        x[nt][0] = v0 ? (sa[nt][0][0] + sa[nt][1][0]) * qs_lo * ks[nt].x : -INFINITY;
        x[nt][1] = v1 ? (sa[nt][0][1] + sa[nt][1][1]) * qs_lo * ks[nt].y : -INFINITY;
        x[nt][2] = v0 ? (sa[nt][0][2] + sa[nt][1][2]) * qs_hi * ks[nt].x : -INFINITY;
        x[nt][3] = v1 ? (sa[nt][0][3] + sa[nt][1][3]) * qs_hi * ks[nt].y : -INFINITY;
        over |= fmaxf(x[nt][0], x[nt][1]) > m_lo + kRescaleThreshold;
        over |= fmaxf(x[nt][2], x[nt][3]) > m_hi + kRescaleThreshold;
      }
      const float kmax = S.kmax[slot];  // the same in every thread
      // The vote barrier also orders this unit's P writes after every warp's
      // P.V of the previous unit (single pair of P tiles).
      const bool vote = named_bar_or(1, NCT, over);
      if (vote || kmax > R) {
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
        const float Rn = fmaxf(R, kmax);
        const float fr = Rn > 0.f ? R / Rn : 0.f;  // O is kept in units of R
        R = Rn;
        invR = R > 0.f ? 1.f / R : 0.f;
        const float o_lo = c_lo * fr, o_hi = c_hi * fr;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          o[nt][0] *= o_lo;
          o[nt][1] *= o_lo;
          o[nt][2] *= o_hi;
          o[nt][3] *= o_hi;
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
          const float p0 = exp2f(x[nt][0] - base_lo), p1 = exp2f(x[nt][1] - base_lo);
          const float p2 = exp2f(x[nt][2] - base_hi), p3 = exp2f(x[nt][3] - base_hi);
          const float w0 = ks[nt].x * invR, w1 = ks[nt].y * invR;
          const uint32_t off_lo = p_chunk(g8, 2 * c + nt) + 4 * q4;
          const uint32_t off_hi = p_chunk(g8 + 8, 2 * c + nt) + 4 * q4;
          sts32(plbase + off_lo, pack_f16x2(p0, p1));
          sts32(plbase + off_hi, pack_f16x2(p2, p3));
          sts32(pvbase + off_lo, pack_f16x2(p0 * w0, p1 * w1));
          sts32(pvbase + off_hi, pack_f16x2(p2 * w0, p3 * w1));
        }
      }
      named_bar(3, NCT);  // P of all 64 keys written

      // ---- O[16 x 128 cols of this warp] += Pv[16 x 64] . V[64 x 128]; l += Pl . 1
      // V words: rows r = 16s + 2q4 + d (d in {0, 1, 8, 9}), chunk
      // ch = 8c + 2Gp + (g8 >> 2), byte 4 (g8 & 3).  With r & 7 = 2q4 + (d & 1)
      // the physical chunk is 8c + 2 (Gp ^ q4) + ((g8 >> 2) ^ (d & 1)): one base
      // register per (d & 1, Gp), the row offset an immediate.
      uint32_t vb[2][4];
#pragma unroll
      for (int d1 = 0; d1 < 2; ++d1)
#pragma unroll
        for (int Gp = 0; Gp < 4; ++Gp)
          vb[d1][Gp] = sb + 2 * q4 * ROW_BYTES +
                       ((8 * c + 2 * (Gp ^ q4) + ((g8 >> 2) ^ d1)) << 4) + 4 * (g8 & 3);
#pragma unroll 1
      for (int s = 0; s < 4; ++s) {  // keys 16s..16s+15 (rolled: bounded loads in flight)
        uint32_t pa[4], pl[4];
        // A-fragments of P for keys 16s..16s+15: chunk 2s + (mtx >> 1)
        const uint32_t pch = p_chunk((lane & 7) + 8 * (mtx & 1), 2 * s + (mtx >> 1));
        ldmatrix_x4(pl, plbase + pch);
        ldmatrix_x4(pa, pvbase + pch);
        mma_f16(lacc, pl, kOnesF16, kOnesF16);
#pragma unroll
        for (int Gp = 0; Gp < 4; ++Gp) {  // columns 128c + 32Gp .. +31
          const uint32_t rs = (uint32_t)(16 * s) * ROW_BYTES;
          const uint32_t wa = lds32(vb[0][Gp] + rs);
          const uint32_t wb = lds32(vb[1][Gp] + rs + ROW_BYTES);
          const uint32_t wc = lds32(vb[0][Gp] + rs + 8 * ROW_BYTES);
          const uint32_t wd = lds32(vb[1][Gp] + rs + 9 * ROW_BYTES);
          uint32_t b0[4], b1[4];  // n-tile j: keys (2q4, 2q4+1) / (2q4+8, 2q4+9), column 4g8 + j
          widen4(__byte_perm(wa, wb, 0x5140), b0[0], b0[1]);
          widen4(__byte_perm(wa, wb, 0x7362), b0[2], b0[3]);
          widen4(__byte_perm(wc, wd, 0x5140), b1[0], b1[1]);
          widen4(__byte_perm(wc, wd, 0x7362), b1[2], b1[3]);
#pragma unroll
          for (int j = 0; j < 4; ++j) mma_f16(o[4 * Gp + j], pa, b0[j], b1[j]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.empty[slot]));  // slot free for the producer

      if (seg_end) {
        // ---------------- epilogue of the segment ending at unit i ----------
        const int64_t tb = t / p.m, tm = t - tb * p.m;
        const float l_lo = lacc[0], l_hi = lacc[2];
        if (kRows || (seg_kb0 == 0 && kb == upt - 1)) {
          const float f_lo = sink_factor(m_lo, l_lo, __ldg(p.sink + g8) * kLog2e) * R;
          const float f_hi = sink_factor(m_hi, l_hi, __ldg(p.sink + g8 + 8) * kLog2e) * R;
          __nv_bfloat16* ob = p.o + tb * p.o_sb + tm * p.o_sm;
#pragma unroll
          for (int Gp = 0; Gp < 4; ++Gp) {
            const int d = 128 * c + 32 * Gp + 8 * q4;
            uint4 lo4, hi4;
            lo4.x = pack_bf16x2(o[4 * Gp + 0][0] * f_lo, o[4 * Gp + 1][0] * f_lo);
            lo4.y = pack_bf16x2(o[4 * Gp + 2][0] * f_lo, o[4 * Gp + 3][0] * f_lo);
            lo4.z = pack_bf16x2(o[4 * Gp + 0][1] * f_lo, o[4 * Gp + 1][1] * f_lo);
            lo4.w = pack_bf16x2(o[4 * Gp + 2][1] * f_lo, o[4 * Gp + 3][1] * f_lo);
            hi4.x = pack_bf16x2(o[4 * Gp + 0][2] * f_hi, o[4 * Gp + 1][2] * f_hi);
            hi4.y = pack_bf16x2(o[4 * Gp + 2][2] * f_hi, o[4 * Gp + 3][2] * f_hi);
            hi4.z = pack_bf16x2(o[4 * Gp + 0][3] * f_hi, o[4 * Gp + 1][3] * f_hi);
            hi4.w = pack_bf16x2(o[4 * Gp + 2][3] * f_hi, o[4 * Gp + 3][3] * f_hi);
            *reinterpret_cast<uint4*>(ob + g8 * p.o_sh + d) = lo4;
            *reinterpret_cast<uint4*>(ob + (g8 + 8) * p.o_sh + d) = hi4;
          }
        } else {
          const int64_t pslot = 2 * g + (t == t_first ? 0 : 1);
          float* pacc = p.part_acc + pslot * kPartAccFloats;
#pragma unroll
          for (int Gp = 0; Gp < 4; ++Gp) {
            const int d = 128 * c + 32 * Gp + 8 * q4;
            float4* lo4 = reinterpret_cast<float4*>(pacc + g8 * kDim + d);
            float4* hi4 = reinterpret_cast<float4*>(pacc + (g8 + 8) * kDim + d);
            lo4[0] = make_float4(o[4 * Gp + 0][0] * R, o[4 * Gp + 1][0] * R,
                                 o[4 * Gp + 2][0] * R, o[4 * Gp + 3][0] * R);
            lo4[1] = make_float4(o[4 * Gp + 0][1] * R, o[4 * Gp + 1][1] * R,
                                 o[4 * Gp + 2][1] * R, o[4 * Gp + 3][1] * R);
            hi4[0] = make_float4(o[4 * Gp + 0][2] * R, o[4 * Gp + 1][2] * R,
                                 o[4 * Gp + 2][2] * R, o[4 * Gp + 3][2] * R);
            hi4[1] = make_float4(o[4 * Gp + 0][3] * R, o[4 * Gp + 1][3] * R,
                                 o[4 * Gp + 2][3] * R, o[4 * Gp + 3][3] * R);
          }
          if (c == 0 && q4 == 0) {
            p.part_ml[pslot * kPartMlFloats + g8] = m_lo;
            p.part_ml[pslot * kPartMlFloats + g8 + 8] = m_hi;
            p.part_ml[pslot * kPartMlFloats + kHeads + g8] = l_lo;
            p.part_ml[pslot * kPartMlFloats + kHeads + g8 + 8] = l_hi;
          }
          if (p.merge_in_kernel) {  // ticket of the split row, as in sa_ws.cu
            const int64_t ts = t * upt;
            const int64_t f = cta_of_unit(ts, p.units, G);
            const int np = static_cast<int>(cta_of_unit(ts + upt - 1, p.units, G) - f + 1);
            __threadfence();
            named_bar(5, NCT);
            if (tt == 0 && atomicAdd(p.tickets + f, 1) == np - 1) {
              p.tickets[f] = 0;
              S.merge_row[S.n_merge++] = t;
            }
          }
        }
      }
      if (seg_end) ++seg;
      seg_first = seg_end;
      if (++kb == nu_t) {
        kb = 0;
        if constexpr (kRows) {
          t = snake_row(++sk, g, G, nrows);
          nu_t = nu_n;
          nu_n = units_of_row(p, snake_row(sk + 1, g, G, nrows));
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
  // ---- every thread merges the split rows whose last part this CTA stored
  __syncthreads();
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

}  // namespace fp8_path

// ---------------------------------------------------------------------------
// Quantiser: bf16 cache rows -> e4m3 rows + one fp32 scale per row.
//   amax = max |x|, y = e4m3_rn_satfinite(x * (448 / amax)), scale = amax / 448
// (amax == 0: y = 0, scale = 0).  One warp per row; lane l holds columns
// 8l..8l+7 and 256+8l..256+8l+7.  HBM-bound: 1 KiB read, 516 B written per row.
// ---------------------------------------------------------------------------
struct QuantParams {
  const __nv_bfloat16* kv;
  uint8_t* kv8;
  float* kscale;
  int64_t b, kv_len;
  int64_t kv_sb, kv_sn, o_sb, o_sn, s_sb, s_sn;
};

__global__ void __launch_bounds__(256) sa_quantize_kv_fp8_kernel(const QuantParams qp) {
  const int64_t rows = qp.b * qp.kv_len;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += warps) {
    const int64_t b = r / qp.kv_len, t = r - b * qp.kv_len;
    const __nv_bfloat16* src = qp.kv + b * qp.kv_sb + t * qp.kv_sn;
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(src + 8 * lane));
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(src + 256 + 8 * lane));
    float v[16];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(v[k]));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float inv = amax > 0.f ? fp8_path::kE4m3Max / amax : 0.f;
    uint32_t y[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      y[k] = (uint32_t)fp8_path::e4m3x2(v[4 * k] * inv, v[4 * k + 1] * inv) |
             ((uint32_t)fp8_path::e4m3x2(v[4 * k + 2] * inv, v[4 * k + 3] * inv) << 16);
    uint8_t* dst = qp.kv8 + b * qp.o_sb + t * qp.o_sn;
    *reinterpret_cast<uint2*>(dst + 8 * lane) = make_uint2(y[0], y[1]);
    *reinterpret_cast<uint2*>(dst + 256 + 8 * lane) = make_uint2(y[2], y[3]);
    if (lane == 0) qp.kscale[b * qp.s_sb + t * qp.s_sn] = amax / fp8_path::kE4m3Max;
  }
}

cudaError_t launch_quantize_fp8(const QuantParams& qp, int sms, cudaStream_t st) {
  const int64_t rows = qp.b * qp.kv_len;
  if (rows == 0) return cudaSuccess;
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)sms * 8;  // 8 resident 256-thread blocks per SM
  if (blocks > cap) blocks = cap;
  sa_quantize_kv_fp8_kernel<<<(unsigned)blocks, 256, 0, st>>>(qp);
  return cudaGetLastError();
}

int read_fp8_error(int* flags) {
  int v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, sa_fp8_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  *flags = v;
  return 0;
}

int reset_fp8_error() {
  const int zero = 0;
  return (int)cudaMemcpyToSymbol(sa_fp8_error, &zero, sizeof(int));
}

int read_fp8_index_faults(unsigned long long* out, bool reset) {
  return index_fault_io(sa_fp8_index_faults, out, reset);
}

int fp8_unit_keys() { return fp8_path::UK; }

cudaError_t encode_q_map(const Params& p, CUtensorMap* q_map);  // sa_tc.cu

cudaError_t launch_fp8(const Params& p, cudaStream_t st) {
  using namespace fp8_path;
  CUtensorMap q_map;
  cudaError_t e = encode_q_map(p, &q_map);
  if (e != cudaSuccess) return e;
  static PerDeviceOnce attr_once;
  e = once_per_device(attr_once, [] {
    const cudaError_t e1 = cudaFuncSetAttribute(
        sa_fp8_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e1 != cudaSuccess) return e1;
    return cudaFuncSetAttribute(sa_fp8_fwd_kernel<true>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
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
  e = cudaLaunchKernelEx(&cfg, rows ? sa_fp8_fwd_kernel<true> : sa_fp8_fwd_kernel<false>, p,
                         q_map);
  if (e != cudaSuccess || p.merge_in_kernel || rows) return e;
  return launch_combine(p, st);
}

}  // namespace sa
