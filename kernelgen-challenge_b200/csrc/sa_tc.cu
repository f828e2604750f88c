// sa_tc.cu — tcgen05 (TMEM accumulator) + TMA-gather variant: not built yet.
#include "sa_common.cuh"

namespace sa {
bool tc_available() { return false; }
int tc_unit_keys() { return 64; }
int tc_ctas_per_sm() { return 1; }
cudaError_t launch_tc(const Params&, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace sa
