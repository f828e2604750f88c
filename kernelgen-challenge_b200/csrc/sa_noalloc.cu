// sa_noalloc.cu — sa_fwd for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: code running inside a
// stream or graph whose memory was reserved up front, plugins whose host
// framework owns every device allocation, or latency-critical serving loops
// that must never enter the allocator.  sa_fwd needs a caller-provided
// workspace for the partial results of query rows that span two persistent
// CTAs; sa_fwd_noalloc instead uses one file-scope device array of fixed size
// that every GPU loading this library holds until the process exits.
//
// The array holds the partials of at most SA_NOALLOC_MAX_CTAS CTAs.  Its
// first bytes are the per-CTA ticket words of the in-kernel merge of split
// rows (prefill-shaped calls without room for the row schedule), which must
// be zero when a call starts: they rely on the zero initialisation of
// __device__ storage when the module loads, and every call leaves them zero
// again (each CTA that takes a ticket still does so when a bounded wait gave
// up, and the last one resets the word).  Everything else in it is written
// before it is read.  All calls on a device share the array, so calls that
// can overlap on that GPU (different streams without ordering between them)
// race and must be serialised by the caller.
#include <mutex>

#include "sa_common.cuh"
#include "sparse_attn.h"

namespace {

constexpr int kMaxCtas = SA_NOALLOC_MAX_CTAS;
constexpr size_t kScratchBytes = sa::workspace_bytes_for_grid(kMaxCtas);
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices];
cudaError_t g_scratch_err[kMaxDevices];
std::once_flag g_scratch_once[kMaxDevices];

}  // namespace

extern "C" int sa_fwd_noalloc(const void* q, const void* kv, const float* sink,
                              const int32_t* idx, void* o, int64_t b, int64_t m, int64_t h,
                              int64_t d, int64_t kv_len, int64_t topk,
                              const int64_t q_strides[4], const int64_t kv_strides[3],
                              const int64_t idx_strides[3], const int64_t o_strides[4],
                              float scale, void* stream, int grid_ctas) {
  if (grid_ctas > kMaxCtas) return SA_ERR_WORKSPACE;  // scratch holds kMaxCtas CTAs
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SA_ERR_CUDA;
  // Once per device, with that device current: the device address of the
  // array (its name in host code is only a host-side stand-in).
  std::call_once(g_scratch_once[dev], [dev] {
    void* ptr = nullptr;
    g_scratch_err[dev] = cudaGetSymbolAddress(&ptr, g_scratch);
    g_scratch_ptr[dev] = ptr;
  });
  if (g_scratch_err[dev] != cudaSuccess || g_scratch_ptr[dev] == nullptr) return SA_ERR_CUDA;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return SA_ERR_CUDA;
  const int grid = grid_ctas > 0 ? grid_ctas : (sms < kMaxCtas ? sms : kMaxCtas);
  return sa_fwd_ex(q, kv, sink, idx, o, b, m, h, d, kv_len, topk, q_strides, kv_strides,
                   idx_strides, o_strides, scale, g_scratch_ptr[dev], kScratchBytes, stream,
                   SA_VARIANT_AUTO, grid);
}
