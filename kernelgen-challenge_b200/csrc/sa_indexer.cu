// sa_indexer.cu — top-k index producer ("lightning indexer") for sm_100a:
// the step before sparse_attn, which turns index queries and index keys into
// the topk_idxs that sparse_attn consumes.
//
// The reference takes topk_idxs as an input (track-01/requirements.md:1-5)
// and has no indexer.  This follows the published DeepSeek-V3.2 lightning
// indexer; the interface is this library's own (include/sparse_attn.h):
//   score[b, t, s] = sum_j w[b, t, j] * ReLU(q[b, t, j, :] . k[b, s, :])
//     for keys s < len[b, t] (the causal or cache limit), fp32 accumulation
//   topk_idxs[b, t, :] = the topk keys of largest score in ascending index
//     order, ties at the threshold to the lower index, -1 padded when fewer
//     keys are valid.
//
// Kernel 1, the scores: sa_indexer_score_tc_kernel (tcgen05, described at its
// definition) by default; sa_indexer_score_kernel, the warp-MMA version, when
// the weight rows cannot be described by a tensor map.  The latter runs one
// CTA per (query row, 4096-key span),
// 4 warps.  The row's q (H = 64 heads x 128 dims, bf16) sits in shared
// memory; 64-key tiles of k stream through a 2-deep cp.async ring.  Warp w
// computes heads 16w..16w+15 against the tile: 8 n-tiles x 8 k-steps of
// mma.sync m16n8k16 bf16 (fp32 accumulate).  ReLU, the head weights, and a
// sum over its 16 heads reduce the fragments to per-key partial scores.  The
// four warps' partials are added in shared memory and the 64 scores are
// written to a fp32 [b*m, kv_len] buffer.
// Kernel 2, sa_indexer_topk_kernel: one CTA per query row, its scores staged
// in shared memory (rows up to 48 Ki keys), radix select of the topk-th
// largest score over order-preserving uint32 keys (an 11-bit round over the
// row, then 11- and 10-bit rounds over the keys of the selected bin), then a
// compaction pass that writes the selected indices in ascending order.
#include <cstdlib>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "sa_common.cuh"
#include "sa_tc.cuh"

namespace sa {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();  // sa_tc.cu
__device__ int sa_idx_error;  // nonzero after a bounded wait of the tensor-core scorer gave up

namespace idx_path {

constexpr int IH = 64;              // index heads
constexpr int ID = 128;             // index head dim
constexpr int TK = 64;              // keys per tile
constexpr int SPAN = 4096;          // keys per scoring CTA
constexpr int NW = 4;
constexpr int NT = NW * 32;
constexpr int KROW = ID * 2;        // 256-byte k rows
constexpr int Q_BYTES = IH * ID * 2;           // 16 KiB
constexpr int TILE_BYTES = TK * KROW;          // 16 KiB

struct IdxParams {
  const __nv_bfloat16* q;  // [b, m, IH, ID]
  const __nv_bfloat16* k;  // [b, kv_len, ID]
  const float* w;          // [b, m, IH]
  const int32_t* len;      // [b, m] valid keys per query (keys s < len)
  float* score;            // [b*m, kv_len] scratch
  int32_t* out;            // [b, m, topk]
  int64_t b, m, kv_len, topk;
  int64_t q_sb, q_sm, q_sh;
  int64_t k_sb, k_sn;
  int64_t w_sb, w_sm;
  int64_t l_sb, l_sm;
  int64_t o_sb, o_sm;
};

// q / k rows in shared memory: 256-byte rows, 16-byte chunks XOR-swizzled by
// the row (ldmatrix of 8 consecutive rows at one chunk is conflict-free)
__device__ __forceinline__ uint32_t row_chunk(int r, int ch) {
  return r * KROW + ((ch ^ (r & 7)) << 4);
}

struct __align__(128) ScoreSmem {
  uint8_t q[Q_BYTES];
  uint8_t tile[2][TILE_BYTES];
  float part[NW][TK];
  float wts[IH];
};

__global__ void __launch_bounds__(NT) sa_indexer_score_kernel(const IdxParams P) {
  extern __shared__ uint8_t smem_raw[];
  ScoreSmem& S = *reinterpret_cast<ScoreSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                               ~static_cast<uintptr_t>(127));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, q4 = lane & 3;
  const int64_t row = blockIdx.x;
  const int64_t tb = row / P.m, tm = row - tb * P.m;
  int64_t L = __ldg(P.len + tb * P.l_sb + tm * P.l_sm);
  L = L < 0 ? 0 : (L > P.kv_len ? P.kv_len : L);
  const int64_t s0 = (int64_t)blockIdx.y * SPAN;
  float* srow = P.score + row * P.kv_len;
  if (s0 >= L) {  // the whole span is past the limit: -inf scores
    for (int64_t s = s0 + tid; s < s0 + SPAN && s < P.kv_len; s += NT) srow[s] = -INFINITY;
    return;
  }
  const int64_t s1 = s0 + SPAN < L ? s0 + SPAN : L;  // keys of this CTA: [s0, s1)
  const int ntiles = static_cast<int>((s1 - s0 + TK - 1) / TK);
  const uint32_t qbase = smem_u32(S.q);
  {
    const __nv_bfloat16* qr = P.q + tb * P.q_sb + tm * P.q_sm;
    for (int c = tid; c < IH * (ID / 8); c += NT) {
      const int h = c / (ID / 8), ch = c % (ID / 8);
      cp_async16(qbase + row_chunk(h, ch), qr + h * P.q_sh + 8 * ch, 16);
    }
    if (tid < IH) S.wts[tid] = __ldg(P.w + tb * P.w_sb + tm * P.w_sm + tid);
  }
  const __nv_bfloat16* kb = P.k + tb * P.k_sb;
  auto issue = [&](int it, int slot) {
    const uint32_t dst = smem_u32(S.tile[slot]);
    const int64_t base = s0 + (int64_t)it * TK;
    for (int c = tid; c < TK * (ID / 8); c += NT) {
      const int r = c / (ID / 8), ch = c % (ID / 8);
      const int64_t s = base + r;
      const bool v = s < s1;
      cp_async16(dst + row_chunk(r, ch), kb + (v ? s : 0) * P.k_sn + 8 * ch, v ? 16 : 0);
    }
    cp_async_commit();
  };
  issue(0, 0);  // (commits the q copies too)
  for (int it = 0; it < ntiles; ++it) {
    const int slot = it & 1;
    if (it + 1 < ntiles) {
      issue(it + 1, slot ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t tbase = smem_u32(S.tile[slot]);
    // warp w: heads 16w..16w+15 x 64 keys, 8 k-steps of 16 dims
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < ID / 16; ++ks) {
      uint32_t a[4];
      {
        const int h = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(a, qbase + row_chunk(h, 2 * ks + (lane >> 4)));
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // key n-tiles 2np, 2np+1
        uint32_t bfrag[4];
        const int key = 16 * np + (lane & 7) + ((lane >> 4) << 3);
        ldmatrix_x4(bfrag, tbase + row_chunk(key, 2 * ks + ((lane >> 3) & 1)));
        mma_16816(acc[2 * np], a, bfrag[0], bfrag[1]);
        mma_16816(acc[2 * np + 1], a, bfrag[2], bfrag[3]);
      }
    }
    // ReLU, head weights, sum over this warp's 16 heads: lane (g8, q4) holds
    // heads 16w + g8 and 16w + g8 + 8 for keys 8nt + 2q4 + {0, 1}
    const float w_lo = S.wts[16 * warp + g8], w_hi = S.wts[16 * warp + g8 + 8];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float v0 = w_lo * fmaxf(acc[nt][0], 0.f) + w_hi * fmaxf(acc[nt][2], 0.f);
      float v1 = w_lo * fmaxf(acc[nt][1], 0.f) + w_hi * fmaxf(acc[nt][3], 0.f);
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {  // over g8
        v0 += __shfl_xor_sync(0xffffffffu, v0, off);
        v1 += __shfl_xor_sync(0xffffffffu, v1, off);
      }
      if (g8 == 0) {
        S.part[warp][8 * nt + 2 * q4] = v0;
        S.part[warp][8 * nt + 2 * q4 + 1] = v1;
      }
    }
    __syncthreads();
    if (tid < TK) {
      const int64_t s = s0 + (int64_t)it * TK + tid;
      if (s < s1) srow[s] = (S.part[0][tid] + S.part[1][tid]) + (S.part[2][tid] + S.part[3][tid]);
    }
    // (the next iteration's __syncthreads orders these reads before the
    // tile and partial buffers are reused)
  }
  // keys of the span past the limit
  for (int64_t s = s1 + tid; s < s0 + SPAN && s < P.kv_len; s += NT) srow[s] = -INFINITY;
}

// ---------------------------------------------------------------------------
// Tensor-core scorer (default): one persistent CTA per SM walks a contiguous
// range of (row group, 128-key tile) items.  A row group is R consecutive
// query rows of one batch (R = 1 when m = 1, else 4), which share each k tile:
//   D[128 keys x 64R] = K_tile[128 x 128] . [q_r0; ...; q_r(R-1)]^T
// (tcgen05.mma kind::f16, M = 128, N = 64R, fp32 accumulators in TMEM).
// Keys sit on M, so TMEM lane i holds key i with its 64 head scores per row
// in columns: each epilogue thread forms sum_j w_j ReLU(.) for its key alone,
// with no cross-thread reduction.  R = 4 reads each k tile once per four rows
// and runs N = 256 MMAs, about twice the work per instruction cycle of N = 64.
//   warp 0  TMA producer: k tiles (two 64-dim slabs, 128-byte swizzle) into a
//           ring; each group's q (two slabs of R x 64 heads) and weights
//           (R x 64 fp32) into one of two buffers
//   warp 1  MMA issuer (one thread): 8 MMAs per tile into one of two TMEM
//           accumulators; commits free the k slot, hand the accumulator to
//           the epilogue, and free the q buffer after a group's last tile
//   warp 2  TMEM allocation (128R columns)
//   warps 4-7  epilogue: TMEM lane quarter w-4 = keys 32(w-4)..+31 of a tile
// Tiles at or past every row's length limit are not loaded or multiplied;
// keys past a row's limit get -inf.  Every wait is bounded (kSpinLimit): on a
// timeout the CTA records sa_idx_error and its roles walk on idle.
// ---------------------------------------------------------------------------
namespace tcx {
using namespace tc;

constexpr int TKEYS = 128;         // keys per tile (M)
constexpr int KSLAB = TKEYS * 128; // 16 KiB: 128 keys x 64 dims
constexpr int KTILE = 2 * KSLAB;   // 32 KiB

template <int R>
struct Cfg {
  static constexpr int NSTAGE = R == 1 ? 4 : 2;  // k ring depth (R = 4: k mostly from L2)
  static constexpr int QSLAB = R * IH * 128;     // R rows x 64 heads x 64 dims
  static constexpr int QTILE = 2 * QSLAB;
  static constexpr uint32_t kTmemCols = 128 * R; // two accumulators of 64R columns
  // epilogue warps: four (one per TMEM lane quarter) for R = 1; eight for
  // R = 4, the second four taking the odd rows of each group
  static constexpr int NE = R == 1 ? 4 : 8;
  static constexpr int NTX = 128 + 32 * NE;
};

template <int R>
struct __align__(1024) Smem {
  uint8_t ring[Cfg<R>::NSTAGE][KTILE];
  uint8_t q[2][Cfg<R>::QTILE];
  float w[2][R][IH];
  uint64_t full[Cfg<R>::NSTAGE], empty[Cfg<R>::NSTAGE], q_full[2], q_empty[2], acc_full[2],
      acc_empty[2], done;
  uint32_t tmem_base;
  int err;
};
template <int R>
constexpr size_t smem_bytes() { return sizeof(Smem<R>) + 1024; }
static_assert(smem_bytes<1>() <= 227 * 1024 && smem_bytes<4>() <= 227 * 1024,
              "shared memory budget");

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* m, int32_t c0,
                                            int32_t c1, int32_t c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

template <class SmemT>
__device__ __forceinline__ bool wait_or_err(SmemT& S, uint64_t& bar, uint32_t parity, int code) {
  if (*reinterpret_cast<volatile int*>(&S.err) != 0) return false;
  if (mbar_wait(smem_u32(&bar), parity)) return true;
  if (atomicCAS(&S.err, 0, code) == 0) atomicCAS(&sa_idx_error, 0, code);
  return false;
}

// The CTA's items and the group bookkeeping every role repeats identically.
template <int R>
struct Walk {
  int64_t grp, tile, tb, m0;
  int64_t L[R];  // length limit of each row (0 for rows past m)
  int64_t Lmax;
  int r;         // groups started so far in this CTA (buffer r & 1)
  bool first;    // first item of a group in this CTA
  __device__ __forceinline__ void at(const IdxParams& P, int64_t item, int64_t tpr, int64_t gpb,
                                     bool start) {
    const int64_t g = item / tpr;
    first = start || g != grp;
    if (first) {
      if (!start) ++r;
      grp = g;
      tb = g / gpb;
      m0 = (g - tb * gpb) * R;
      Lmax = 0;
#pragma unroll
      for (int k = 0; k < R; ++k) {
        int64_t l = 0;
        if (m0 + k < P.m) {
          l = __ldg(P.len + tb * P.l_sb + (m0 + k) * P.l_sm);
          l = l < 0 ? 0 : (l > P.kv_len ? P.kv_len : l);
        }
        L[k] = l;
        Lmax = l > Lmax ? l : Lmax;
      }
    }
    tile = item - g * tpr;
  }
};

template <int R>
__global__ void __launch_bounds__(Cfg<R>::NTX, 1)
    sa_indexer_score_tc_kernel(const IdxParams P, const __grid_constant__ CUtensorMap k_map,
                               const __grid_constant__ CUtensorMap q_map,
                               const __grid_constant__ CUtensorMap w_map) {
  using C = Cfg<R>;
  constexpr int NS = C::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  Smem<R>& S = *reinterpret_cast<Smem<R>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t tpr = (P.kv_len + TKEYS - 1) / TKEYS;  // tiles per group
  const int64_t gpb = (P.m + R - 1) / R;               // groups per batch
  const int64_t items = P.b * gpb * tpr;
  const int64_t G = gridDim.x, g = blockIdx.x;
  const int64_t i0 = (g * items) / G, i1 = ((g + 1) * items) / G;
  const int n = static_cast<int>(i1 - i0);
  if (n <= 0) return;
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&S.full[s]), 1);
      mbar_init(smem_u32(&S.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&S.q_full[b]), 1);
      // freed by the MMA commit after a group's last tile and by the
      // epilogue warps (they read the group's weights from the buffer)
      mbar_init(smem_u32(&S.q_empty[b]), 1 + C::NE);
      mbar_init(smem_u32(&S.acc_full[b]), 1);
      mbar_init(smem_u32(&S.acc_empty[b]), C::NE);
    }
    mbar_init(smem_u32(&S.done), 1);
    S.err = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc<C::kTmemCols>(smem_u32(&S.tmem_base));
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&k_map);
    tma_prefetch_desc(&q_map);
    tma_prefetch_desc(&w_map);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      Walk<R> w{};
      for (int i = 0; i < n; ++i) {
        w.at(P, i0 + i, tpr, gpb, i == 0);
        if (w.first) {
          const int qb = w.r & 1;
          if (w.r < 2 || wait_or_err(S, S.q_empty[qb], ((w.r >> 1) - 1) & 1, 1)) {
            mbar_arrive_expect_tx(smem_u32(&S.q_full[qb]), C::QTILE + R * IH * 4);
            for (int sl = 0; sl < 2; ++sl)
              tma_load_4d(smem_u32(S.q[qb]) + sl * C::QSLAB, &q_map, 64 * sl, 0, (int32_t)w.m0,
                          (int32_t)w.tb, smem_u32(&S.q_full[qb]));
            tma_load_3d(smem_u32(&S.w[qb][0][0]), &w_map, 0, (int32_t)w.m0, (int32_t)w.tb,
                        smem_u32(&S.q_full[qb]));
          }
        }
        const int slot = i % NS;
        if (i >= NS && !wait_or_err(S, S.empty[slot], ((i / NS) - 1) & 1, 2)) continue;
        if (w.tile * TKEYS < w.Lmax) {
          mbar_arrive_expect_tx(smem_u32(&S.full[slot]), KTILE);
          for (int sl = 0; sl < 2; ++sl)
            tma_load_3d(smem_u32(S.ring[slot]) + sl * KSLAB, &k_map, 64 * sl,
                        (int32_t)(w.tile * TKEYS), (int32_t)w.tb, smem_u32(&S.full[slot]));
        } else {
          mbar_arrive(smem_u32(&S.full[slot]));  // nothing to load: keys past every limit
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(TKEYS, IH * R, false, false);
      Walk<R> w{};
      for (int i = 0; i < n; ++i) {
        w.at(P, i0 + i, tpr, gpb, i == 0);
        const int qb = w.r & 1, slot = i % NS, ab = i & 1;
        const bool last_of_group = (i == n - 1) || (w.tile == tpr - 1);
        bool ok = !w.first || wait_or_err(S, S.q_full[qb], (w.r >> 1) & 1, 3);
        ok = ok && wait_or_err(S, S.full[slot], (i / NS) & 1, 4);
        ok = ok && (i < 2 || wait_or_err(S, S.acc_empty[ab], ((i >> 1) - 1) & 1, 5));
        if (!ok) continue;
        tc_fence_after();
        if (w.tile * TKEYS < w.Lmax) {
          const uint32_t kb = smem_u32(S.ring[slot]), qa = smem_u32(S.q[qb]);
#pragma unroll
          for (int sl = 0; sl < 2; ++sl)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16_ss(tmem + IH * R * ab,
                         smem_desc(kb + sl * KSLAB + kk * 32, 16, 1024, kLayoutSw128),
                         smem_desc(qa + sl * C::QSLAB + kk * 32, 16, 1024, kLayoutSw128), idesc,
                         (sl | kk) != 0);
        }
        mma_commit(smem_u32(&S.empty[slot]));
        mma_commit(smem_u32(&S.acc_full[ab]));
        if (last_of_group) mma_commit(smem_u32(&S.q_empty[qb]));
      }
      // every MMA of this thread complete before TMEM is released
      mma_commit(smem_u32(&S.done));
      mbar_wait(smem_u32(&S.done), 0);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // --------------------------------------------------------------- epilogue
    constexpr int RSTEP = C::NE / 4;  // rows per group step of one warp
    const int qd = (warp - 4) & 3, half = (warp - 4) >> 2;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * qd) << 16);
    Walk<R> w{};
    for (int i = 0; i < n; ++i) {
      w.at(P, i0 + i, tpr, gpb, i == 0);
      const int ab = i & 1, qb = w.r & 1;
      // (warp-uniform: tcgen05.ld below is a warp-wide instruction)
      bool ok = __all_sync(0xffffffffu, wait_or_err(S, S.acc_full[ab], (i >> 1) & 1, 6));
      // the group's weights landed with its q (the MMA waited for them)
      if (w.first) ok = ok && __all_sync(0xffffffffu, wait_or_err(S, S.q_full[qb], (w.r >> 1) & 1, 7));
      tc_fence_after();
      const int64_t key = w.tile * TKEYS + 32 * qd + lane;
      const bool active = ok && w.tile * TKEYS < w.Lmax;
#pragma unroll
      for (int kk = 0; kk < R; kk += RSTEP) {
        // row k = kk + half (RSTEP = 2) or kk (RSTEP = 1); the length limit is
        // picked without indexing L by a run-time value
        const int k = kk + (RSTEP == 2 ? half : 0);
        const int64_t Lk = (RSTEP == 2 && half) ? w.L[(kk + 1) % R] : w.L[kk];
        if (w.m0 + k >= P.m) break;
        float score = -INFINITY;
        if (active && w.tile * TKEYS < Lk) {
          float v[4][16];  // the row's 64 head scores of this key, one wait
#pragma unroll
          for (int c = 0; c < IH / 16; ++c)
            tmem_ld16(lane_addr + IH * R * ab + IH * k + 16 * c, v[c]);
          tmem_wait_ld();
          const float* wt = S.w[qb][k];
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int c = 0; c < IH / 16; ++c)
#pragma unroll
            for (int e = 0; e < 16; ++e)
              acc[c] = fmaf(wt[16 * c + e], fmaxf(v[c][e], 0.f), acc[c]);
          if (key < Lk) score = (acc[0] + acc[1]) + (acc[2] + acc[3]);
        }
        const int64_t row = w.tb * P.m + w.m0 + k;
        if (key < P.kv_len) P.score[row * P.kv_len + key] = score;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&S.acc_empty[ab]));
        if (i == n - 1 || w.tile == tpr - 1) mbar_arrive(smem_u32(&S.q_empty[qb]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc<C::kTmemCols>(tmem);
  }
}

}  // namespace tcx

// ---------------------------------------------------------------------------
// Top-k of one row of scores: the topk-th largest key by radix select
// (coalesced histogram passes), then an ordered compaction in which warp w
// owns a contiguous block of keys, read 32 at a time, with ballots giving the
// output positions.  The output row is contiguous.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t order_key(float x) {  // larger float -> larger key
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Rows of up to kSmemKeys scores are staged in shared memory once; the
// histogram rounds and the compaction then read them there (longer rows read
// the fp32 score buffer, L2-resident, every time).
constexpr int kSmemKeys = 49152;  // 192 KiB

// Inclusive prefix sum over the block (NT threads); `scratch` holds NT/32 ints.
template <int NT>
__device__ __forceinline__ int block_incl_scan(int v, int* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += y;
  }
  if (lane == 31) scratch[wid] = inc;
  __syncthreads();
  int before = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) before += w < wid ? scratch[w] : 0;
  __syncthreads();  // scratch reused by the next scan
  return before + inc;
}

// One radix round over n keys (get(i) -> order key): among the keys whose
// bits under `pmask` equal `prefix`, histogram the BITS-bit digit at `shift`
// (warp-aggregated shared-memory adds: most keys share few digits), then find
// the digit holding rank kk counted from the largest.  Returns the digit and
// leaves in kk the rank still to find among the keys with that digit.
template <int NT, int BITS, class Get>
__device__ __forceinline__ uint32_t radix_round(Get get, int n, uint32_t prefix, uint32_t pmask,
                                                int shift, int& kk, int* hist, int* scratch,
                                                int* sh) {
  constexpr int NB = 1 << BITS, BPT = (NB + NT - 1) / NT;
  const int tid = threadIdx.x;
  for (int d = tid; d < NB; d += NT) hist[d] = 0;
  __syncthreads();
  for (int base = 0; base < n; base += NT) {
    const int i = base + tid;
    uint32_t d = NB;  // no bin
    if (i < n) {
      const uint32_t key = get(i);
      if ((key & pmask) == prefix) d = (key >> shift) & (NB - 1);
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    if (d < NB && (__ffs(peers) - 1) == (tid & 31)) atomicAdd(&hist[d], __popc(peers));
  }
  __syncthreads();
  // thread t owns bins NB-1-t*BPT down to NB-(t+1)*BPT: counts from the top
  int c = 0;
#pragma unroll
  for (int e = 0; e < BPT; ++e) {
    const int b = NB - 1 - tid * BPT - e;
    if (b >= 0) c += hist[b];
  }
  const int inc = block_incl_scan<NT>(c, scratch);
  const int before = inc - c;
  if (before < kk && kk <= inc) {
    int acc = before;
    for (int e = 0; e < BPT; ++e) {
      const int b = NB - 1 - tid * BPT - e;
      if (acc + hist[b] >= kk) {
        sh[0] = b;
        sh[1] = kk - acc;
        break;
      }
      acc += hist[b];
    }
  }
  __syncthreads();
  const uint32_t digit = static_cast<uint32_t>(sh[0]);
  kk = sh[1];
  __syncthreads();  // hist and sh reused by the next round
  return digit;
}

// NT2 threads per row: 1024 for long rows (one row per SM: the row's staged
// scores fill its shared memory, and the rounds' barrier chains need every
// warp the SM can hold), 128 for rows of up to kShortRow keys, so that more
// rows run side by side.
// Selection: an 11-bit round over the whole row (sign, exponent and three
// mantissa bits of the scores) finds the bin holding the topk-th largest key;
// that bin's keys are gathered into a short candidate list, and two more
// rounds (11 and 10 bits) over the list give the exact threshold key.  A bin
// too large for the list runs those rounds over the whole row instead.
constexpr int kShortRow = 8192;
template <int NT2>
constexpr int cand_cap() { return NT2 == 128 ? 1024 : 4096; }

template <int NT2>
__global__ void __launch_bounds__(NT2, 1) sa_indexer_topk_kernel(const IdxParams P) {
  extern __shared__ float staged[];
  __shared__ int hist[2048];
  __shared__ uint32_t cand[cand_cap<NT2>()];
  __shared__ int scratch[NT2 / 32];
  __shared__ int sh[2];
  __shared__ int cand_n;
  __shared__ int sel_rem;
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int64_t tb = row / P.m, tm = row - tb * P.m;
  int64_t L = __ldg(P.len + tb * P.l_sb + tm * P.l_sm);
  L = L < 0 ? 0 : (L > P.kv_len ? P.kv_len : L);
  const float* srow = P.score + row * P.kv_len;
  if (P.kv_len <= kSmemKeys) {
    if ((P.kv_len & 3) == 0) {  // 16-byte rows: float4 copies, four per thread in flight
      const int64_t n4 = (L + 3) / 4;
      for (int64_t v = tid; v < n4; v += NT2)
        reinterpret_cast<float4*>(staged)[v] = __ldg(reinterpret_cast<const float4*>(srow) + v);
    } else {
      for (int64_t s = tid; s < L; s += NT2) staged[s] = srow[s];
    }
    srow = staged;
  }
  if (tid == 0) cand_n = 0;
  __syncthreads();
  int32_t* orow = P.out + tb * P.o_sb + tm * P.o_sm;
  const int64_t K = P.topk;

  // threshold key T and the number of keys equal to T that are taken
  uint32_t T = 0;
  int take_eq = 0;
  const bool all = L <= K;  // every valid key is selected
  if (!all) {
    const int n = static_cast<int>(L);
    auto row_key = [&](int i) { return order_key(srow[i]); };
    int kk = static_cast<int>(K);  // rank still to find among keys matching the prefix
    const uint32_t b0 = radix_round<NT2, 11>(row_key, n, 0u, 0u, 21, kk, hist, scratch, sh);
    const uint32_t p0 = b0 << 21, m0 = 0x7FFu << 21;
    // gather the keys of bin b0 (order does not matter for the threshold)
    for (int base = 0; base < n; base += NT2) {
      const int i = base + tid;
      const uint32_t key = i < n ? row_key(i) : 0u;
      const bool in = i < n && (key & m0) == p0;
      const uint32_t bal = __ballot_sync(0xffffffffu, in);
      int at = 0;
      if ((tid & 31) == 0 && bal != 0) at = atomicAdd(&cand_n, __popc(bal));
      at = __shfl_sync(0xffffffffu, at, 0) + __popc(bal & ((1u << (tid & 31)) - 1u));
      if (in && at < cand_cap<NT2>()) cand[at] = key;
    }
    __syncthreads();
    const int nc = cand_n;
    uint32_t b1, b2;
    if (nc <= cand_cap<NT2>()) {
      auto cand_key = [&](int i) { return cand[i]; };
      b1 = radix_round<NT2, 11>(cand_key, nc, p0, m0, 10, kk, hist, scratch, sh);
      b2 = radix_round<NT2, 10>(cand_key, nc, p0 | (b1 << 10), m0 | (0x7FFu << 10), 0, kk, hist,
                                scratch, sh);
    } else {
      b1 = radix_round<NT2, 11>(row_key, n, p0, m0, 10, kk, hist, scratch, sh);
      b2 = radix_round<NT2, 10>(row_key, n, p0 | (b1 << 10), m0 | (0x7FFu << 10), 0, kk, hist,
                                scratch, sh);
    }
    T = p0 | (b1 << 10) | b2;
    take_eq = kk;  // keys equal to T to take, lowest indices first
  }
  // Ordered compaction.  Warp w owns the contiguous keys [w*C, (w+1)*C), read
  // 32 at a time (lane-consecutive, so shared memory is conflict-free); the
  // keys equal to T are taken lowest index first, take_eq of them.
  const int wid = tid >> 5, ln = tid & 31;
  constexpr int NWARP = NT2 / 32;
  if (all) {
    for (int64_t s = tid; s < L; s += NT2) orow[s] = static_cast<int32_t>(s);
    for (int64_t j = L + tid; j < K; j += NT2) orow[j] = -1;
    return;
  }
  const int Ci = (int)(((L + NWARP - 1) / NWARP + 31) / 32 * 32);
  const int c0 = wid * Ci, c1 = (c0 + Ci < (int)L) ? c0 + Ci : (int)L;
  int n_gt = 0, n_eq = 0;
  for (int s = c0 + ln; s < c1; s += 32) {
    const uint32_t key = order_key(srow[s]);
    n_gt += key > T;
    n_eq += key == T;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    n_gt += __shfl_xor_sync(0xffffffffu, n_gt, off);
    n_eq += __shfl_xor_sync(0xffffffffu, n_eq, off);
  }
  __shared__ int w_eq[NWARP], w_sel[NWARP];
  if (ln == 0) w_eq[wid] = n_eq;
  __syncthreads();
  if (wid == 0) {  // per warp: keys equal to T before it, then selected keys before it
    int e = ln < NWARP ? w_eq[ln] : 0;
    int inc = e;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, inc, off);
      if (ln >= off) inc += y;
    }
    const int eq_before = inc - e;
    if (ln < NWARP) w_eq[ln] = eq_before;
  }
  __syncthreads();
  int eq_seen = w_eq[wid];  // keys equal to T before this warp's next block
  const int eq_take = max(0, min(n_eq, take_eq - eq_seen));
  if (ln == 0) w_sel[wid] = n_gt + eq_take;
  __syncthreads();
  if (wid == 0) {
    int e = ln < NWARP ? w_sel[ln] : 0;
    int inc = e;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, inc, off);
      if (ln >= off) inc += y;
    }
    if (ln < NWARP) w_sel[ln] = inc - e;
    if (ln == NWARP - 1) sel_rem = inc;  // selected keys in all
  }
  __syncthreads();
  int pos = w_sel[wid];
  const int n_total = sel_rem;
  const uint32_t lt = (1u << ln) - 1u;
  for (int s0 = c0; s0 < c1; s0 += 32) {
    const int s = s0 + ln;
    const uint32_t key = s < c1 ? order_key(srow[s]) : 0u;
    const bool eq = s < c1 && key == T;
    const uint32_t beq = __ballot_sync(0xffffffffu, eq);
    const bool take = (s < c1 && key > T) || (eq && eq_seen + __popc(beq & lt) < take_eq);
    const uint32_t bt = __ballot_sync(0xffffffffu, take);
    if (take) orow[pos + __popc(bt & lt)] = static_cast<int32_t>(s);
    pos += __popc(bt);
    eq_seen += __popc(beq);
  }
  for (int64_t j = n_total + tid; j < K; j += NT2) orow[j] = -1;
}

}  // namespace idx_path

namespace {

cudaError_t launch_score_tc(const idx_path::IdxParams& P, const int64_t q_strides[4],
                            const int64_t k_strides[3], const int64_t w_strides[3],
                            cudaStream_t st) {
  using namespace idx_path::tcx;
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return cudaErrorNotSupported;
  const int R = P.m == 1 ? 1 : 4;
  CUtensorMap k_map, q_map, w_map;
  {  // k [b, kv_len, 128]: boxes of 64 dims x 128 keys, 128-byte swizzle
    cuuint64_t dims[3] = {128, (cuuint64_t)P.kv_len, (cuuint64_t)P.b};
    cuuint64_t strides[2] = {(cuuint64_t)k_strides[1] * 2, (cuuint64_t)k_strides[0] * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)TKEYS, 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(&k_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16*>(P.k), dims,
            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {  // q [b, m, 64, 128]: boxes of 64 dims x 64 heads x R rows (rows past m read zeros)
    cuuint64_t dims[4] = {128, (cuuint64_t)idx_path::IH, (cuuint64_t)P.m, (cuuint64_t)P.b};
    cuuint64_t strides[3] = {(cuuint64_t)q_strides[2] * 2, (cuuint64_t)q_strides[1] * 2,
                             (cuuint64_t)q_strides[0] * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)idx_path::IH, (cuuint32_t)R, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&q_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<__nv_bfloat16*>(P.q), dims,
            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {  // weights [b, m, 64] fp32: boxes of 64 x R rows
    cuuint64_t dims[3] = {(cuuint64_t)idx_path::IH, (cuuint64_t)P.m, (cuuint64_t)P.b};
    cuuint64_t strides[2] = {(cuuint64_t)w_strides[1] * 4, (cuuint64_t)w_strides[0] * 4};
    cuuint32_t box[3] = {(cuuint32_t)idx_path::IH, (cuuint32_t)R, 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(&w_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(P.w), dims, strides,
            box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  auto* kern = R == 1 ? sa_indexer_score_tc_kernel<1> : sa_indexer_score_tc_kernel<4>;
  const size_t smem = R == 1 ? smem_bytes<1>() : smem_bytes<4>();
  static PerDeviceOnce attr_once;
  cudaError_t e = once_per_device(attr_once, [] {
    const cudaError_t e1 =
        cudaFuncSetAttribute(sa_indexer_score_tc_kernel<1>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes<1>());
    if (e1 != cudaSuccess) return e1;
    return cudaFuncSetAttribute(sa_indexer_score_tc_kernel<4>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem_bytes<4>());
  });
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int64_t items = P.b * ((P.m + R - 1) / R) * ((P.kv_len + TKEYS - 1) / TKEYS);
  const int64_t grid = items < sms ? items : sms;
  kern<<<static_cast<unsigned>(grid), R == 1 ? Cfg<1>::NTX : Cfg<4>::NTX, smem, st>>>(
      P, k_map, q_map, w_map);
  return cudaGetLastError();
}

}  // namespace

int read_indexer_error(int* flags) {
  int v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, sa_idx_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  *flags = v;
  return 0;
}

int reset_indexer_error() {
  const int zero = 0;
  return (int)cudaMemcpyToSymbol(sa_idx_error, &zero, sizeof(int));
}

cudaError_t launch_indexer(const __nv_bfloat16* q, const __nv_bfloat16* k, const float* w,
                           const int32_t* len, int32_t* out, float* score, int64_t b, int64_t m,
                           int64_t kv_len, int64_t topk, const int64_t q_strides[4],
                           const int64_t k_strides[3], const int64_t w_strides[3],
                           const int64_t len_strides[2], const int64_t out_strides[3],
                           cudaStream_t st) {
  using namespace idx_path;
  IdxParams P{q, k, w, len, score, out, b, m, kv_len, topk,
              q_strides[0], q_strides[1], q_strides[2], k_strides[0], k_strides[1],
              w_strides[0], w_strides[1], len_strides[0], len_strides[1],
              out_strides[0], out_strides[1]};
  static PerDeviceOnce attr_once;
  const size_t smem = sizeof(ScoreSmem) + 128;
  cudaError_t e = once_per_device(attr_once, [&] {
    cudaError_t e1 = cudaFuncSetAttribute(sa_indexer_score_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e1 != cudaSuccess) return e1;
    e1 = cudaFuncSetAttribute(sa_indexer_topk_kernel<128>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)(kShortRow * sizeof(float)));
    if (e1 != cudaSuccess) return e1;
    return cudaFuncSetAttribute(sa_indexer_topk_kernel<1024>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(kSmemKeys * sizeof(float)));
  });
  if (e != cudaSuccess) return e;
  const int64_t rows = P.b * P.m;
  const int64_t spans = (P.kv_len + SPAN - 1) / SPAN;
  if (spans > 0) {  // (no keys: the top-k kernel writes -1 everywhere)
    // the tensor maps need 16-byte-aligned weight rows (q and k rows are
    // checked by the caller); otherwise the warp-MMA scorer runs
    const bool w_ok = (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && w_strides[0] % 4 == 0 &&
                      w_strides[1] % 4 == 0;
    if (sa::opt_indexer_tc() && w_ok) {
      e = launch_score_tc(P, q_strides, k_strides, w_strides, st);
    } else {
      sa_indexer_score_kernel<<<dim3(static_cast<unsigned>(rows), static_cast<unsigned>(spans)),
                                NT, smem, st>>>(P);
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) return e;
  }
  const size_t staged = kv_len <= kSmemKeys ? (size_t)kv_len * sizeof(float) : 0;
  if (kv_len <= kShortRow) {
    sa_indexer_topk_kernel<128><<<static_cast<unsigned>(rows), 128, staged, st>>>(P);
  } else {
    sa_indexer_topk_kernel<1024><<<static_cast<unsigned>(rows), 1024, staged, st>>>(P);
  }
  return cudaGetLastError();
}

}  // namespace sa
