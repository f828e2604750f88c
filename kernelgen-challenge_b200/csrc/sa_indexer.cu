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
// Kernel 1, sa_indexer_score_kernel: one CTA per (query row, 4096-key span),
// 4 warps.  The row's q (H = 64 heads x 128 dims, bf16) sits in shared
// memory; 64-key tiles of k stream through a 2-deep cp.async ring.  Warp w
// computes heads 16w..16w+15 against the tile: 8 n-tiles x 8 k-steps of
// mma.sync m16n8k16 bf16 (fp32 accumulate).  ReLU, the head weights, and a
// sum over its 16 heads reduce the fragments to per-key partial scores.  The
// four warps' partials are added in shared memory and the 64 scores are
// written to a fp32 [b*m, kv_len] buffer.
// Kernel 2, sa_indexer_topk_kernel: one CTA per query row, its scores staged
// in shared memory (rows up to 48 Ki keys), radix select of the topk-th
// largest score over order-preserving uint32 keys (four 8-bit histogram
// rounds), then a compaction pass that writes the selected indices in
// ascending order.
#include "sa_common.cuh"

namespace sa {
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
// Top-k of one row of scores: the topk-th largest key by radix select
// (coalesced histogram passes), then an ordered compaction in which thread t
// owns the contiguous keys [t*seg, (t+1)*seg).  The output row is contiguous.
// ---------------------------------------------------------------------------
constexpr int NT2 = 512;

__device__ __forceinline__ uint32_t order_key(float x) {  // larger float -> larger key
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive prefix sum over the block (NT2 threads); returns the block total.
__device__ __forceinline__ int block_excl_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += y;
  }
  if (lane == 31) warp_sums[wid] = inc;
  __syncthreads();
  if (wid == 0) {
    int w = lane < NT2 / 32 ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    if (lane < NT2 / 32) warp_sums[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int before = (wid > 0 ? warp_sums[wid - 1] : 0) + inc - v;
  total = warp_sums[NT2 / 32 - 1];
  __syncthreads();  // warp_sums reused by the next scan
  return before;
}

// Rows of up to kSmemKeys scores are staged in shared memory once; the four
// histogram rounds and the compaction then read them there (longer rows read
// the fp32 score buffer, L2-resident, every time).
constexpr int kSmemKeys = 49152;  // 192 KiB

__global__ void __launch_bounds__(NT2) sa_indexer_topk_kernel(const IdxParams P) {
  extern __shared__ float staged[];
  __shared__ int hist[256];
  __shared__ int warp_sums[32];
  __shared__ uint32_t sel_digit;
  __shared__ int sel_rem;
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int64_t tb = row / P.m, tm = row - tb * P.m;
  int64_t L = __ldg(P.len + tb * P.l_sb + tm * P.l_sm);
  L = L < 0 ? 0 : (L > P.kv_len ? P.kv_len : L);
  const float* srow = P.score + row * P.kv_len;
  if (P.kv_len <= kSmemKeys) {
    for (int64_t s = tid; s < L; s += NT2) staged[s] = srow[s];
    __syncthreads();
    srow = staged;
  }
  int32_t* orow = P.out + tb * P.o_sb + tm * P.o_sm;
  const int64_t K = P.topk;
  const int64_t seg = (L + NT2 - 1) / NT2;
  const int64_t a0 = tid * seg, a1 = (a0 + seg < L) ? a0 + seg : L;

  // threshold key T and the number of keys equal to T that are taken
  uint32_t T = 0;
  int take_eq = 0;
  const bool all = L <= K;  // every valid key is selected
  if (!all) {
    uint32_t prefix = 0, pmask = 0;
    int kk = static_cast<int>(K);  // rank still to find among keys matching prefix
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int d = tid; d < 256; d += NT2) hist[d] = 0;
      __syncthreads();
      // coalesced pass (order does not matter here); warp-aggregated adds,
      // since most keys share the leading digits
      for (int64_t base = 0; base < L; base += NT2) {
        const int64_t s = base + tid;
        uint32_t d = 256;  // no bin
        if (s < L) {
          const uint32_t key = order_key(srow[s]);
          if ((key & pmask) == prefix) d = (key >> shift) & 255;
        }
        const uint32_t peers = __match_any_sync(0xffffffffu, d);
        if (d < 256 && (__ffs(peers) - 1) == (tid & 31)) atomicAdd(&hist[d], __popc(peers));
      }
      __syncthreads();
      if (tid < 32) {  // scan the 256 bins from the top: bin holding rank kk
        // lane l covers bins 255-8l .. 248-8l
        int c = 0;
        for (int e = 0; e < 8; ++e) c += hist[255 - 8 * tid - e];
        int inc = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, inc, off);
          if (tid >= off) inc += y;
        }
        const int before = inc - c;
        const bool mine = before < kk && kk <= inc;
        if (mine) {
          int acc = before;
          for (int e = 0; e < 8; ++e) {
            const int d = 255 - 8 * tid - e;
            if (acc + hist[d] >= kk) {
              sel_digit = static_cast<uint32_t>(d);
              sel_rem = kk - acc;
              break;
            }
            acc += hist[d];
          }
        }
      }
      __syncthreads();
      prefix |= sel_digit << shift;
      pmask |= 255u << shift;
      kk = sel_rem;
      __syncthreads();
    }
    T = prefix;
    take_eq = kk;  // keys equal to T to take, lowest indices first
  }
  // ordered compaction: ties before this thread's segment, then positions
  int n_gt = 0, n_eq = 0;
  if (!all) {
    for (int64_t s = a0; s < a1; ++s) {
      const uint32_t key = order_key(srow[s]);
      n_gt += key > T;
      n_eq += key == T;
    }
  }
  int tot;
  const int eq_before = block_excl_scan(n_eq, warp_sums, tot);
  const int eq_mine = all ? 0 : max(0, min(n_eq, take_eq - eq_before));
  const int n_sel = all ? static_cast<int>(a1 > a0 ? a1 - a0 : 0) : n_gt + eq_mine;
  int n_total;
  int pos = block_excl_scan(n_sel, warp_sums, n_total);
  int eq_used = 0;
  for (int64_t s = a0; s < a1; ++s) {
    bool take;
    if (all) {
      take = true;
    } else {
      const uint32_t key = order_key(srow[s]);
      take = key > T || (key == T && eq_used < eq_mine);
      eq_used += key == T;
    }
    if (take) orow[pos++] = static_cast<int32_t>(s);
  }
  for (int64_t j = n_total + tid; j < K; j += NT2) orow[j] = -1;
}

}  // namespace idx_path

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
    return cudaFuncSetAttribute(sa_indexer_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(kSmemKeys * sizeof(float)));
  });
  if (e != cudaSuccess) return e;
  const int64_t rows = P.b * P.m;
  const int64_t spans = (P.kv_len + SPAN - 1) / SPAN;
  if (spans > 0) {  // (no keys: the top-k kernel writes -1 everywhere)
    sa_indexer_score_kernel<<<dim3(static_cast<unsigned>(rows), static_cast<unsigned>(spans)),
                              NT, smem, st>>>(P);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const size_t staged = kv_len <= kSmemKeys ? (size_t)kv_len * sizeof(float) : 0;
  sa_indexer_topk_kernel<<<static_cast<unsigned>(rows), NT2, staged, st>>>(P);
  return cudaGetLastError();
}

}  // namespace sa
