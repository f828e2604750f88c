// sa_bwd.cu — backward pass of sparse_attn for sm_100a: gradients of q, the
// KV cache and the sink, given o and dO from the forward.
//
// The reference has no backward.  This restates the gradient of its forward
// (track-01/reference/reference.py:24-40, masking of
// track-01/submission.py:313-322).  Per query row and head h, with p_t the
// softmax weights over the valid slots and the sink, and v_t = k_t = kv[idx_t]:
//   D      = sum_d dO . o                    (o from the forward)
//   dp_t   = dO . v_t
//   ds_t   = p_t (dp_t - D)
//   dq     = scale * sum_t ds_t k_t
//   dkv[idx_t] += scale * ds_t q + p_t dO    (summed over heads; duplicates add)
//   dsink  = -p_sink * D                     (summed over rows)
//
// One CTA (8 warps, two per SM sub-partition) per query row.  Its units of 64
// gathered rows, up to the last unit holding a valid slot (the forward's
// 128-byte-swizzled slab layout), stream through a 2-deep cp.async ring twice
// (once when the training forward supplied the log-sum-exp):
//   pass A  S = Q.K^T (warp w: keys 8w..8w+7), online max / sum per head: the
//           row's log-sum-exp including the sink
//   pass B  S and dP = dO.V^T again (warp w: keys 8w..8w+7), P and
//           dS = P (dP - D) * scale into shared memory (bf16), then
//           dq[16 x 64w..64w+63] += dS . K   (registers, whole row)
//           dkv [16 keys of group w & 3 x 256 columns of half w >> 2]
//             = dS^T . Q + P^T . dO in 64-column chunks, staged in shared
//             memory and added into an fp32 gradient buffer by TMA bulk
//             reductions, 256 bytes per key (masked slots skip)
// All products are bf16 warp MMAs with fp32 accumulation.
#include "sa_common.cuh"

namespace sa {
namespace bwd_path {

constexpr int UK = 64;                      // keys per unit
constexpr int NW = 8;                       // warps
constexpr int NT = NW * 32;
constexpr int SLOT_BYTES = UK * kDim * 2;   // 64 KiB
constexpr int SLAB_BYTES = UK * 128;        // [64 keys x 64 cols]
constexpr int T_BYTES = kHeads * kDim * 2;  // 16 KiB: Q or dO tile
constexpr int P_BYTES = kHeads * UK * 2;    // 2 KiB: P or dS tile [head][key]

struct BwdParams {
  Params f;                  // forward arguments (q, kv, sink, idx, o, shapes, strides)
  const __nv_bfloat16* dout; // dO, strides as o
  __nv_bfloat16* dq;         // rows of [16, 512], dq_rs elements apart
  int64_t dq_rs;
  float* dkv;                // [b, kv_len, 512] fp32, row stride dkv_sn
  float* dsink;              // [16] fp32
  int64_t dkv_sb, dkv_sn;
  float scale;
  // kSplit instance: each row's units are cut into `splits` contiguous parts,
  // CTA x running part x % splits of row x / splits (one pass: lse given);
  // the parts add dq into dq_acc (fp32, zero-filled, rows dq_rs floats apart)
  int splits;
  float* dq_acc;
};

struct __align__(1024) Smem {
  uint8_t ring[2][SLOT_BYTES];
  uint8_t q[T_BYTES];   // 8 slabs [16 heads][64 cols], chunks swizzled by head
  uint8_t dout[T_BYTES];
  uint8_t p[P_BYTES];   // P   [head][key] bf16, chunks swizzled
  uint8_t ds[P_BYTES];  // dS * scale
  int32_t ids[2][UK];   // slot ids of the unit in each ring slot (-1: masked)
  float red[NW][2][kHeads];
  float D[kHeads];
  float M[kHeads];      // log2-domain max including the sink
  float invZ[kHeads];
  // per warp: its [16 keys x 64 cols] fp32 dkv chunk, rows padded to 288 bytes
  // (the fragment stores of a half-warp hit 32 distinct banks), read by the
  // bulk reductions
  float dk[NW][16][72];
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

__device__ __forceinline__ uint32_t p_chunk(int h, int ch) {
  return h * 128 + ((ch ^ (h & 7)) << 4);
}
// byte offset of the 16-byte chunk holding columns 8c..8c+7 of head h in a Q / dO tile
__device__ __forceinline__ uint32_t t_chunk(int h, int c) {
  return (c >> 3) * 2048 + h * 128 + (((c & 7) ^ (h & 7)) << 4);
}

// dst[0..bytes) += src (fp32, element-wise, in L2), by the TMA unit; both
// addresses 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_reduce_add_f32(float* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;\n" ::"l"(
                   dst),
               "r"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
}
// all but this thread's newest N bulk-operation groups have finished
// reading shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
// ... and are complete
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void sts64f(uint32_t addr, float a, float b) {
  asm volatile("st.shared.v2.f32 [%0], {%1,%2};\n" ::"r"(addr), "f"(a), "f"(b) : "memory");
}

template <bool kSplit>
__global__ void __launch_bounds__(NT, 1) sa_bwd_kernel(const BwdParams bp) {
  extern __shared__ uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
  const Params& p = bp.f;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, q4 = lane & 3;
  const int64_t row = kSplit ? blockIdx.x / bp.splits : blockIdx.x;
  const int64_t tb = row / p.m, tm = row - tb * p.m;
  const int32_t* irow = p.idx + tb * p.i_sb + tm * p.i_sm;
  // Units up to the row's last valid slot: trailing masked slots (causal
  // prefill pads each row with -1) are neither gathered nor multiplied.  One
  // CTA per row, so the GPU's own block scheduling balances short rows.
  __shared__ int64_t units_s;
  if (warp == 0) {
    int64_t last = -1;
    for (int64_t base = ((p.topk - 1) / 32) * 32; base >= 0; base -= 32) {
      const int64_t k = base + lane;
      const int32_t id = k < p.topk ? __ldg(irow + k * p.i_sk) : -1;
      const uint32_t v = __ballot_sync(0xffffffffu, id >= 0 && (int64_t)id < p.kv_len);
      if (v != 0u) {
        last = base + 31 - __clz(v);
        break;
      }
    }
    if (lane == 0) units_s = (last + UK) / UK;  // ceil((last + 1) / UK)
  }
  __syncthreads();
  const int64_t U = units_s;
  const __nv_bfloat16* kvb = p.kv + tb * p.kv_sb;
  const uint32_t qbase = smem_u32(S.q), dobase = smem_u32(S.dout);
  const uint32_t pbase = smem_u32(S.p), dsbase = smem_u32(S.ds);

  // ---- Q and dO of this row into their tiles; D = dO . o per head
  {
    const __nv_bfloat16* qr = p.q + tb * p.q_sb + tm * p.q_sm;
    const __nv_bfloat16* dr = bp.dout + tb * p.o_sb + tm * p.o_sm;
    for (int k = tid; k < kHeads * (kDim / 8); k += NT) {  // 16-byte chunks
      const int h = k / (kDim / 8), c = k % (kDim / 8);
      cp_async16(qbase + t_chunk(h, c), qr + h * p.q_sh + 8 * c, 16);
      cp_async16(dobase + t_chunk(h, c), dr + h * p.o_sh + 8 * c, 16);
    }
    cp_async_commit();
    const __nv_bfloat16* orow = p.o + tb * p.o_sb + tm * p.o_sm;
    for (int h = warp; h < kHeads; h += NW) {
      float acc = 0.f;
      for (int c = lane; c < kDim / 8; c += 32) {
        const uint4 a = *reinterpret_cast<const uint4*>(orow + h * p.o_sh + 8 * c);
        const uint4 d = *reinterpret_cast<const uint4*>(dr + h * p.o_sh + 8 * c);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, dw[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&aw[e]));
          const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dw[e]));
          acc += x.x * y.x + x.y * y.y;
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      if (lane == 0) S.D[h] = acc;
    }
  }

  // ---- gather of unit u into ring slot s: thread copies chunk tid & 63 of
  // rows (tid >> 6) + 4k
  auto issue = [&](int64_t u, int s) {
    const int c = tid & 63, par = tid >> 6, j = c >> 3, cc = c & 7;
    const uint32_t dst0 = smem_u32(S.ring[s]) + j * SLAB_BYTES;
    for (int k = 0; k < UK / 4; ++k) {
      const int r = par + 4 * k;
      const int64_t key = u * UK + r;
      const int32_t id = key < p.topk ? __ldg(irow + key * p.i_sk) : -1;
      const bool v = id >= 0 && (int64_t)id < p.kv_len;
      cp_async16(dst0 + r * 128 + ((cc ^ (r & 7)) << 4), kvb + (v ? (int64_t)id : 0) * p.kv_sn + c * 8,
                 v ? 16 : 0);
      if (c == 0) S.ids[s][r] = v ? id : -1;
    }
    cp_async_commit();
  };

  // S (or dP with the dO tile) for keys 8w..8w+7: sa[z] split accumulators
  // (even / odd k-steps)
  auto scores = [&](uint32_t sb, uint32_t abase, float (&sa)[2][4]) {
#pragma unroll
    for (int z = 0; z < 2; ++z) sa[z][0] = sa[z][1] = sa[z][2] = sa[z][3] = 0.f;
    const int arow = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll 4
    for (int kp = 0; kp < 16; ++kp) {  // columns 32kp..32kp+31
      uint32_t a0[4], a1[4];
      ldmatrix_x4(a0, abase + t_chunk(arow, 4 * kp + (lane >> 4)));
      ldmatrix_x4(a1, abase + t_chunk(arow, 4 * kp + 2 + (lane >> 4)));
      const int slab = kp >> 1, c0 = (kp & 1) * 4;
      const int key = 8 * warp + (lane & 7);
      uint32_t kf[4];
      ldmatrix_x4(kf, sb + slab * SLAB_BYTES + key * 128 + (((c0 + (lane >> 3)) ^ (key & 7)) << 4));
      mma_16816(sa[0], a0, kf[0], kf[1]);
      mma_16816(sa[1], a1, kf[2], kf[3]);
    }
  };

  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;  // pass A, this lane's keys
  float dq[8][4];  // dq[heads g8, g8+8][64w + 8nt + 2q4 + {0,1}]
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) dq[nt][0] = dq[nt][1] = dq[nt][2] = dq[nt][3] = 0.f;

  // with the forward's log-sum-exp (sa_fwd_train) pass A is skipped; the
  // loop runs i = i0 .. iend - 1, unit i % U (i >= U: pass B)
  int64_t i0 = p.lse != nullptr ? U : 0, iend = 2 * U;
  if constexpr (kSplit) {  // (lse given)
    const int64_t part = blockIdx.x % bp.splits;
    i0 = U + part * U / bp.splits;
    iend = U + (part + 1) * U / bp.splits;
  }
  if (p.lse != nullptr && tid < kHeads) {
    const float sl2 = __ldg(p.sink + tid) * kLog2e;
    const float L = p.lse[row * p.lse_rs + tid];
    S.M[tid] = L;
    S.invZ[tid] = 1.f;
    // dsink = -p_sink * D once the D of this row is in shared memory (below)
    S.red[0][0][tid] = exp2f(sl2 - L);
  }
  if (i0 < iend) issue(i0 % U, i0 & 1);
  if (p.lse != nullptr) {
    __syncthreads();  // D and the sink weights
    if (tid < kHeads && (!kSplit || blockIdx.x % bp.splits == 0))
      atomicAdd(bp.dsink + tid, -S.red[0][0][tid] * S.D[tid]);
  }
  for (int64_t i = i0; i < iend; ++i) {
    const int s = static_cast<int>(i & 1);
    if (i + 1 < iend) {
      issue((i + 1) % U, s ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // unit i landed (and, at i = 0, the Q / dO tiles and D)
    const uint32_t sb = smem_u32(S.ring[s]);
    const bool passB = i >= U;
    if (i == U && i0 == 0) {
      // ---- end of pass A: M and 1/Z per head, including the sink
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        const float mo_lo = __shfl_xor_sync(0xffffffffu, m_lo, off);
        const float lo_lo = __shfl_xor_sync(0xffffffffu, l_lo, off);
        const float mo_hi = __shfl_xor_sync(0xffffffffu, m_hi, off);
        const float lo_hi = __shfl_xor_sync(0xffffffffu, l_hi, off);
        const float n_lo = fmaxf(m_lo, mo_lo), n_hi = fmaxf(m_hi, mo_hi);
        l_lo = (n_lo == -INFINITY) ? 0.f : l_lo * exp2f(m_lo - n_lo) + lo_lo * exp2f(mo_lo - n_lo);
        l_hi = (n_hi == -INFINITY) ? 0.f : l_hi * exp2f(m_hi - n_hi) + lo_hi * exp2f(mo_hi - n_hi);
        m_lo = n_lo;
        m_hi = n_hi;
      }
      if (q4 == 0) {
        S.red[warp][0][g8] = m_lo;
        S.red[warp][1][g8] = l_lo;
        S.red[warp][0][g8 + 8] = m_hi;
        S.red[warp][1][g8 + 8] = l_hi;
      }
      __syncthreads();
      if (tid < kHeads) {
        const float sl2 = __ldg(p.sink + tid) * kLog2e;
        float M = sl2;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, S.red[w][0][tid]);
        float Z = exp2f(sl2 - M);
        for (int w = 0; w < NW; ++w)
          if (S.red[w][0][tid] != -INFINITY) Z += S.red[w][1][tid] * exp2f(S.red[w][0][tid] - M);
        S.M[tid] = M;
        S.invZ[tid] = 1.f / Z;
        // dsink = -p_sink * D
        atomicAdd(bp.dsink + tid, -exp2f(sl2 - M) / Z * S.D[tid]);
      }
      __syncthreads();
    }
    float sa[2][4];
    scores(sb, qbase, sa);
    float x[4];  // [0,1] head g8, [2,3] head g8+8; keys 8w + 2q4 + {0,1}
    {
      const int key = 8 * warp + 2 * q4;
      const bool v0 = S.ids[s][key] >= 0, v1 = S.ids[s][key + 1] >= 0;
      x[0] = v0 ? (sa[0][0] + sa[1][0]) * p.scale_log2 : -INFINITY;
      x[1] = v1 ? (sa[0][1] + sa[1][1]) * p.scale_log2 : -INFINITY;
      x[2] = v0 ? (sa[0][2] + sa[1][2]) * p.scale_log2 : -INFINITY;
      x[3] = v1 ? (sa[0][3] + sa[1][3]) * p.scale_log2 : -INFINITY;
    }
    if (!passB) {
      // online max / sum of this lane's keys
      const float n_lo = fmaxf(m_lo, fmaxf(x[0], x[1])), n_hi = fmaxf(m_hi, fmaxf(x[2], x[3]));
      if (n_lo != -INFINITY) {
        l_lo = l_lo * exp2f(m_lo - n_lo) + exp2f(x[0] - n_lo) + exp2f(x[1] - n_lo);
        m_lo = n_lo;
      }
      if (n_hi != -INFINITY) {
        l_hi = l_hi * exp2f(m_hi - n_hi) + exp2f(x[2] - n_hi) + exp2f(x[3] - n_hi);
        m_hi = n_hi;
      }
      __syncthreads();  // slot s free for the next issue
      continue;
    }
    // ---- pass B: P, dP, dS
    float dpa[2][4];
    scores(sb, dobase, dpa);
    {
      const float M_lo = S.M[g8], M_hi = S.M[g8 + 8];
      const float iz_lo = S.invZ[g8], iz_hi = S.invZ[g8 + 8];
      const float D_lo = S.D[g8], D_hi = S.D[g8 + 8];
      const float p0 = exp2f(x[0] - M_lo) * iz_lo, p1 = exp2f(x[1] - M_lo) * iz_lo;
      const float p2 = exp2f(x[2] - M_hi) * iz_hi, p3 = exp2f(x[3] - M_hi) * iz_hi;
      const float d0 = p0 * (dpa[0][0] + dpa[1][0] - D_lo) * bp.scale;
      const float d1 = p1 * (dpa[0][1] + dpa[1][1] - D_lo) * bp.scale;
      const float d2 = p2 * (dpa[0][2] + dpa[1][2] - D_hi) * bp.scale;
      const float d3 = p3 * (dpa[0][3] + dpa[1][3] - D_hi) * bp.scale;
      *reinterpret_cast<uint32_t*>(S.p + p_chunk(g8, warp) + 4 * q4) = pack_bf16x2(p0, p1);
      *reinterpret_cast<uint32_t*>(S.p + p_chunk(g8 + 8, warp) + 4 * q4) = pack_bf16x2(p2, p3);
      *reinterpret_cast<uint32_t*>(S.ds + p_chunk(g8, warp) + 4 * q4) = pack_bf16x2(d0, d1);
      *reinterpret_cast<uint32_t*>(S.ds + p_chunk(g8 + 8, warp) + 4 * q4) = pack_bf16x2(d2, d3);
    }
    __syncthreads();  // P and dS of all 64 keys written
    // ---- dq[16 x 64w..64w+63] += dS[16 x 64] . K[64 x 64] (slab w)
#pragma unroll
    for (int kst = 0; kst < 4; ++kst) {
      uint32_t da[4];
      {
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(da, dsbase + p_chunk(r, 2 * kst + (lane >> 4)));
      }
      const int kr = kst * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int ch = (np << 1) + (lane >> 4);
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, sb + warp * SLAB_BYTES + kr * 128 + ((ch ^ (kr & 7)) << 4));
        mma_16816(dq[2 * np], da, vb[0], vb[1]);
        mma_16816(dq[2 * np + 1], da, vb[2], vb[3]);
      }
    }
    // ---- dkv[keys 16kg..16kg+15][columns 256ch..+255] = dS^T . Q + P^T . dO,
    //      64 columns at a time (kg = w & 3, ch = w >> 2)
    {
      const int kg = warp & 3, chh = warp >> 2;
      // A-fragments (rows = keys, k = heads) by transposed loads of the
      // [head][key] tiles: matrices (heads 0-7 | 8-15) x (keys 16kg..+7 | 16kg+8..+15)
      const int mt = lane >> 3, hr = (lane & 7) + 8 * (mt >> 1), kc = 2 * kg + (mt & 1);
      uint32_t ad[4], ap[4];
      ldmatrix_x4_trans(ad, dsbase + p_chunk(hr, kc));
      ldmatrix_x4_trans(ap, pbase + p_chunk(hr, kc));
      // lanes 0..15 add key 16kg + lane's row of each chunk
      const int32_t id_mine = lane < 16 ? S.ids[s][16 * kg + lane] : -1;
      float* drow = bp.dkv + tb * bp.dkv_sb + (int64_t)(id_mine < 0 ? 0 : id_mine) * bp.dkv_sn;
      const uint32_t stage = smem_u32(&S.dk[warp][0][0]);
      // B-fragments (k = heads, n = columns) by transposed loads of the Q / dO
      // tiles: matrices (heads 0-7 | 8-15) x (columns n0..n0+7 | n0+8..n0+15)
      const int br = (lane & 7) + 8 * (mt & 1), bcol = (mt >> 1);
#pragma unroll 1
      for (int cb = 4 * chh; cb < 4 * chh + 4; ++cb) {
        float acc[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // n-tiles 2np, 2np+1: columns 64cb + 16np ..
          uint32_t bq[4], bd[4];
          const int c8 = 8 * cb + 2 * np + bcol;
          ldmatrix_x4_trans(bq, qbase + t_chunk(br, c8));
          ldmatrix_x4_trans(bd, dobase + t_chunk(br, c8));
          mma_16816(acc[2 * np], ad, bq[0], bq[1]);
          mma_16816(acc[2 * np + 1], ad, bq[2], bq[3]);
          mma_16816(acc[2 * np], ap, bd[0], bd[1]);
          mma_16816(acc[2 * np + 1], ap, bd[2], bd[3]);
        }
        // the chunk to the warp's stage (once the previous chunk's reductions
        // have read it), then one 256-byte bulk reduction per valid key.
        // (Two 128-byte stages, one filled while the other's reductions run,
        // were slower: the reductions' cost grows with their count.)
        bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const uint32_t c4 = (8 * nt + 2 * q4) * 4;
          sts64f(stage + g8 * 288 + c4, acc[nt][0], acc[nt][1]);
          sts64f(stage + (g8 + 8) * 288 + c4, acc[nt][2], acc[nt][3]);
        }
        fence_proxy_async_smem();  // the stores precede the reductions' reads
        __syncwarp();
        if (id_mine >= 0) {
          bulk_reduce_add_f32(drow + 64 * cb, stage + lane * 288, 256);
          bulk_commit();
        }
      }
    }
    __syncthreads();  // slot s and the P / dS tiles free
  }
  cp_async_wait<0>();  // (no units: the Q / dO copies)
  bulk_wait();         // the dkv reductions are done before the CTA exits
  // ---- dq of this row (the scale is already in dS)
  if constexpr (kSplit) {  // this part's share, added into the fp32 rows
    if (iend > i0) {
      float* dqa = bp.dq_acc + row * bp.dq_rs;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int d = 64 * warp + 8 * nt + 2 * q4;
        atomicAdd(reinterpret_cast<float2*>(dqa + g8 * kDim + d), make_float2(dq[nt][0], dq[nt][1]));
        atomicAdd(reinterpret_cast<float2*>(dqa + (g8 + 8) * kDim + d),
                  make_float2(dq[nt][2], dq[nt][3]));
      }
    }
    return;
  }
  __nv_bfloat16* dqr = bp.dq + row * bp.dq_rs;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int d = 64 * warp + 8 * nt + 2 * q4;
    *reinterpret_cast<uint32_t*>(dqr + g8 * kDim + d) = pack_bf16x2(dq[nt][0], dq[nt][1]);
    *reinterpret_cast<uint32_t*>(dqr + (g8 + 8) * kDim + d) = pack_bf16x2(dq[nt][2], dq[nt][3]);
  }
}

// ---------------------------------------------------------------------------
// The rows of a dense KV gradient that one call touches: the kv rows its
// valid slots name.  Decode-shaped calls touch far fewer rows than the cache
// holds (b = 64 x 2048 slots of a 32,768-row cache), so the fp32 buffer the
// backward kernel adds into is zeroed, and cast to bf16, on those rows only.
// One warp per (b, m, slot); each instruction of the warp covers 512
// contiguous bytes of the row.  Duplicated indices repeat the same stores.
struct RowsParams {
  float* dkv;                // fp32 [b][kv_len][512], strides dkv_sb, dkv_sn
  __nv_bfloat16* out;        // kCast: bf16 rows, strides out_sb, out_sn
  const int32_t* idx;
  int64_t b, m, topk, kv_len;
  int64_t i_sb, i_sm, i_sk, dkv_sb, dkv_sn, out_sb, out_sn;
};

template <bool kCast>
__global__ void __launch_bounds__(256) sa_dkv_rows_kernel(const RowsParams rp) {
  const int lane = threadIdx.x & 31;
  const int64_t nslot = rp.b * rp.m * rp.topk;
  for (int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); w < nslot;
       w += (int64_t)gridDim.x * 8) {
    const int64_t r = w / rp.topk, k = w - r * rp.topk;
    const int64_t tb = r / rp.m, tm = r - tb * rp.m;
    const int32_t id = __ldg(rp.idx + tb * rp.i_sb + tm * rp.i_sm + k * rp.i_sk);
    if (id < 0 || (int64_t)id >= rp.kv_len) continue;  // masked: no row touched
    float4* row = reinterpret_cast<float4*>(rp.dkv + tb * rp.dkv_sb + (int64_t)id * rp.dkv_sn);
    if constexpr (kCast) {
      uint2* orow = reinterpret_cast<uint2*>(rp.out + tb * rp.out_sb + (int64_t)id * rp.out_sn);
      float4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = __ldcg(row + lane + 32 * j);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        orow[lane + 32 * j] = make_uint2(pack_bf16x2(v[j].x, v[j].y), pack_bf16x2(v[j].z, v[j].w));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) row[lane + 32 * j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// dq[row][h][:] = bf16(dq_acc[row][h][:]) for the 16 heads of a group
__global__ void __launch_bounds__(256) sa_dq_cast_kernel(const float* acc, __nv_bfloat16* dq,
                                                         int64_t rows, int64_t rs) {
  const int64_t n4 = rows * (kHeads * kDim / 4);
  for (int64_t k = (int64_t)blockIdx.x * 256 + threadIdx.x; k < n4; k += (int64_t)gridDim.x * 256) {
    const int64_t r = k / (kHeads * kDim / 4), c = (k - r * (kHeads * kDim / 4)) * 4;
    const float4 v = __ldcg(reinterpret_cast<const float4*>(acc + r * rs + c));
    *reinterpret_cast<uint2*>(dq + r * rs + c) =
        make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

}  // namespace bwd_path

cudaError_t launch_dkv_rows(bool cast, float* dkv, __nv_bfloat16* out, const int32_t* idx,
                            int64_t b, int64_t m, int64_t topk, int64_t kv_len,
                            const int64_t idx_strides[3], const int64_t dkv_strides[3],
                            const int64_t out_strides[3], int sms, cudaStream_t st) {
  bwd_path::RowsParams rp{dkv, out, idx, b, m, topk, kv_len,
                idx_strides[0], idx_strides[1], idx_strides[2], dkv_strides[0], dkv_strides[1],
                cast ? out_strides[0] : 0, cast ? out_strides[1] : 0};
  const int64_t nslot = b * m * topk;
  if (nslot == 0) return cudaSuccess;
  int64_t blocks = (nslot + 7) / 8;
  if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
  if (cast) {
    bwd_path::sa_dkv_rows_kernel<true><<<static_cast<unsigned>(blocks), 256, 0, st>>>(rp);
  } else {
    bwd_path::sa_dkv_rows_kernel<false><<<static_cast<unsigned>(blocks), 256, 0, st>>>(rp);
  }
  return cudaGetLastError();
}

cudaError_t launch_bwd(const Params& f, const __nv_bfloat16* dout, __nv_bfloat16* dq,
                       int64_t dq_rs, float* dkv, float* dsink, int64_t dkv_sb, int64_t dkv_sn,
                       float scale, float* dq_acc, int sms, cudaStream_t st) {
  using namespace bwd_path;
  static PerDeviceOnce attr_once;
  cudaError_t e = once_per_device(attr_once, [] {
    const cudaError_t e1 = cudaFuncSetAttribute(
        sa_bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e1 != cudaSuccess) return e1;
    return cudaFuncSetAttribute(sa_bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  const int64_t rows = f.b * f.m;
  // Fewer rows than SMs (decode): with the log-sum-exp and an fp32 dq
  // scratch, each row runs as `splits` parts on as many CTAs, one wave in
  // all (the kernel holds one CTA per SM); each part keeps >= 2 units.
  int splits = 1;
  if (dq_acc != nullptr && f.lse != nullptr && rows > 0 && rows * 2 <= sms) {
    splits = static_cast<int>(sms / rows);
    const int64_t max_parts = (f.topk + 2 * UK - 1) / (2 * UK);
    if (splits > max_parts) splits = static_cast<int>(max_parts > 1 ? max_parts : 1);
  }
  BwdParams bp{f, dout, dq, dq_rs, dkv, dsink, dkv_sb, dkv_sn, scale, splits, dq_acc};
  if (splits == 1) {  // the kernel writes dq itself; dq_acc, if given, stays unused
    sa_bwd_kernel<false><<<static_cast<unsigned>(rows), NT, kSmemBytes, st>>>(bp);
    return cudaGetLastError();
  }
  sa_bwd_kernel<true><<<static_cast<unsigned>(rows * splits), NT, kSmemBytes, st>>>(bp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int64_t blocks = (rows * (kHeads * kDim / 4) + 255) / 256;
  if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
  sa_dq_cast_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(dq_acc, dq, rows, dq_rs);
  return cudaGetLastError();
}

}  // namespace sa
