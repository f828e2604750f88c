// sa_probe.cu — the random-row gather on its own: the copy side of the
// sparse_attn kernels with no math, to measure how fast this B200 serves
// scattered rows of a KV cache (sa_probe_gather, include/sparse_attn.h).
//
// Every CTA walks a contiguous share of a row list in 32 KiB units (the rows
// of one unit land in one ring slot of shared memory, or in registers) and
// does nothing with the data beyond folding one word per thread into a
// checksum, so the time is the gather alone.  Three copy forms:
//   0  cp.async 16 B per thread (the forward kernels' form): 128 producer
//      threads, L2 evict_first hint, completion by cp.async.mbarrier.arrive;
//   1  cp.async.bulk (1-D TMA, one CTA), one bulk copy per row, issued by
//      the 32 lanes of one warp, completion by the mbarrier's byte count;
//   2  ld.global.nc 16 B into registers, 256 threads, 8 loads in flight each.
// Forms 0 and 1 use a ring of `depth` slots with one consumer warp that waits
// for a slot, reads a word and frees it.  Every wait is bounded: on a timeout
// the kernel records an error in *err and stops issuing copies.
#include "sa_tc.cuh"
#include "sparse_attn.h"

namespace sa {
namespace probe {
using namespace tc;

constexpr int NT = 256;
constexpr int SLOT = 32768;
constexpr int MAX_DEPTH = 6;

struct Params {
  const uint8_t* src;
  const int32_t* rows;
  int64_t n_rows, row_stride;  // bytes between rows of src
  int row_bytes, method, depth;
  int cpr_log2;  // log2(16-byte chunks per row)
  int ids_offset;  // byte offset of the staged row indices in dynamic shared memory
  uint32_t* sink;
  int* err;
};

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ uint4 ldg_nc16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity, volatile int* err) {
  if (*err != 0) return false;
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && *err != 0) return false;
  }
  atomicCAS(const_cast<int*>(err), 0, 1);
  return false;
}

__global__ void __launch_bounds__(NT) probe_gather_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)p.depth * SLOT);
  uint64_t* empty = full + MAX_DEPTH;
  __shared__ int s_err;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rows_per_unit = SLOT / p.row_bytes;
  const int64_t units = (p.n_rows + rows_per_unit - 1) / rows_per_unit;
  const int64_t u0 = blockIdx.x * units / gridDim.x, u1 = (blockIdx.x + 1) * units / gridDim.x;
  const int n = static_cast<int>(u1 - u0);
  const int cpr_mask = (1 << p.cpr_log2) - 1;
  uint32_t acc = 0;
  // The CTA's row indices, staged in shared memory up front (one round trip),
  // so that no copy waits on an index load: the time is the gather alone.
  int32_t* ids = reinterpret_cast<int32_t*>(smem_raw + p.ids_offset);
  const int64_t r_begin = u0 * rows_per_unit;
  const int n_ids = static_cast<int>(min((int64_t)n * rows_per_unit, p.n_rows - r_begin));
  for (int k = tid; k < n_ids; k += NT) ids[k] = __ldg(p.rows + r_begin + k);
  __syncthreads();

  if (p.method == 2) {  // registers: each thread owns 8 chunks of every unit
    for (int i = 0; i < n; ++i) {
      const int64_t r0 = (u0 + i) * rows_per_unit;
      uint4 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int c = tid + k * NT;
        const int64_t r = r0 + (c >> p.cpr_log2);
        const int64_t row = r < p.n_rows ? ids[r - r_begin] : 0;
        v[k] = ldg_nc16(p.src + row * p.row_stride + (c & cpr_mask) * 16);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) acc ^= v[k].x ^ v[k].w;
    }
    if (acc == 0x9e3779b9u) atomicXor(p.sink + blockIdx.x, acc);  // keeps the loads live
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < p.depth; ++s) {
      mbar_init(smem_u32(&full[s]), p.method == 0 ? 128 : 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    s_err = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* err = &s_err;
  if (warp < 4) {
    const uint64_t pol = l2_policy_evict_first();
    for (int i = 0; i < n; ++i) {
      const int slot = i % p.depth;
      const bool ok = i < p.depth ||
                      bounded_wait(smem_u32(&empty[slot]), ((i / p.depth) - 1) & 1, err);
      if (!ok) continue;
      const int64_t r0 = (u0 + i) * rows_per_unit;
      const uint32_t dst = smem_u32(ring + (size_t)slot * SLOT);
      if (p.method == 0) {
#pragma unroll 4
        for (int c = tid; c < SLOT / 16; c += 128) {
          const int64_t r = r0 + (c >> p.cpr_log2);
          const bool v = r < p.n_rows;
          const int64_t row = v ? ids[r - r_begin] : 0;
          cp_async16_hint(dst + c * 16, p.src + row * p.row_stride + (c & cpr_mask) * 16,
                          v ? 16 : 0, pol);
        }
        cp_async_mbar_arrive_noinc(smem_u32(&full[slot]));
      } else if (warp == 0) {
        const uint32_t bar = smem_u32(&full[slot]);
        if (lane == 0) mbar_arrive_expect_tx(bar, SLOT);
        __syncwarp();
        for (int k = lane; k < rows_per_unit; k += 32) {
          const int64_t r = r0 + k;
          const int64_t row = r < p.n_rows ? ids[r - r_begin] : ids[0];
          bulk_g2s(dst + k * p.row_bytes, p.src + row * p.row_stride, p.row_bytes, bar);
        }
      }
    }
    if (p.method == 0) cp_async_wait<0>();
  } else if (warp == 4) {
    for (int i = 0; i < n; ++i) {
      const int slot = i % p.depth;
      if (bounded_wait(smem_u32(&full[slot]), (i / p.depth) & 1, err))
        acc ^= reinterpret_cast<const uint32_t*>(ring + (size_t)slot * SLOT)[lane * 97];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty[slot]));
    }
    if (acc == 0x9e3779b9u) atomicXor(p.sink + blockIdx.x, acc);
  }
  __syncthreads();
  // bulk copies still in flight after an error: wait for the slots' byte
  // counts to drain (bounded) before the CTA's shared memory is released
  if (*err != 0 && p.method == 1 && tid == 0) {
    for (int s = 0; s < p.depth && s < n; ++s) {
      const int last = s + ((n - 1 - s) / p.depth) * p.depth;  // last unit in slot s
      for (uint32_t k = 0; k < kSpinLimit && !mbar_try_wait(smem_u32(&full[s]), (last / p.depth) & 1);
           ++k) {
      }
    }
  }
  if (tid == 0 && *err != 0) atomicCAS(p.err, 0, 1);
}

}  // namespace probe
}  // namespace sa

extern "C" int sa_probe_gather(const void* src, int64_t row_stride, const int32_t* rows,
                               int64_t n_rows, int64_t row_bytes, int method, int ctas, int depth,
                               uint32_t* sink, int* err, void* stream) {
  using namespace sa::probe;
  if (!src || !rows || !sink || !err || n_rows < 0) return SA_ERR_INVALID_ARG;
  if (row_bytes < 16 || row_bytes > SLOT || (row_bytes & (row_bytes - 1)) != 0)
    return SA_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0 || (row_stride % 16) != 0 ||
      row_stride < row_bytes)
    return SA_ERR_INVALID_ARG;
  if (method < 0 || method > 2 || ctas < 1 || ctas > 4096 || depth < 2 || depth > MAX_DEPTH)
    return SA_ERR_INVALID_ARG;
  if (n_rows == 0) return SA_OK;
  int lg = 0;
  while ((16 << lg) < row_bytes) ++lg;
  Params p{static_cast<const uint8_t*>(src), rows, n_rows, row_stride, static_cast<int>(row_bytes),
           method, depth, lg, 0, sink, err};
  // per CTA: its share of the units, rounded up, in indices (4 B each)
  const int64_t rpu = SLOT / row_bytes;
  const int64_t units = (n_rows + rpu - 1) / rpu;
  const int64_t ids_bytes = ((units + ctas - 1) / ctas) * rpu * 4;
  const size_t ring = method == 2 ? 0 : (size_t)depth * SLOT + 2 * MAX_DEPTH * 8 + 128;
  p.ids_offset = static_cast<int>(ring);
  const size_t smem = ring + (size_t)ids_bytes;
  if (smem > 227 * 1024) return SA_ERR_INVALID_ARG;
  cudaError_t e = cudaFuncSetAttribute(probe_gather_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return SA_ERR_CUDA;
  probe_gather_kernel<<<ctas, NT, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? SA_OK : SA_ERR_CUDA;
}
